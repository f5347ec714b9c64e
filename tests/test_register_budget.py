"""Register budgets that set occupancy, checked from ptxas's report on the CPU (nvcc
cross-compiles for sm_100a without a GPU).

The B = 512 decode streams 2.16 GB of state per step and reaches the HBM rate only with
three 256-thread CTAs per SM in flight: at 86 registers the two-rows-per-thread instance
dropped to two CTAs per SM and the step went from 0.32 to 0.37 ms.  These checks catch such
a change before it reaches a GPU."""
import os
import re
import shutil
import subprocess

import pytest

from fastaf_kernel_b200 import build as B

NVCC = shutil.which("nvcc") or ("/usr/local/cuda/bin/nvcc" if os.path.exists("/usr/local/cuda/bin/nvcc") else None)
pytestmark = pytest.mark.skipif(NVCC is None, reason="nvcc not available")


def _ptxas_report(source: str, tmp_path):
    """{mangled kernel name: (registers, spill store bytes, spill load bytes)} for one source."""
    cmd = [NVCC, "-c", os.path.join(B.CSRC, source), "-o", str(tmp_path / "k.o")] + B.ARCH_FLAGS + [
        "-O3", "-std=c++17", "-I", B.INCLUDE, "-I", B.CSRC, "--expt-relaxed-constexpr", "-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    out, name, spills = {}, None, (0, 0)
    for line in r.stderr.splitlines():
        m = re.search(r"Compiling entry function '([^']+)'", line)
        if m:
            name, spills = m.group(1), (0, 0)
            continue
        m = re.search(r"(\d+) bytes spill stores, (\d+) bytes spill loads", line)
        if m and name:
            spills = (int(m.group(1)), int(m.group(2)))
            continue
        m = re.search(r"Used (\d+) registers", line)
        if m and name:
            out[name] = (int(m.group(1)), *spills)
            name = None
    return out


def test_decode_instances_keep_three_ctas_per_sm(tmp_path):
    rep = _ptxas_report("gdn_decode.cu", tmp_path)
    dec = {k: v for k, v in rep.items() if "decode_kernel" in k}
    assert len(dec) == 4, sorted(rep)          # rows per thread 1, 2 x q/k normalisation off, on
    for name, (regs, st, ld) in dec.items():
        # 65,536 registers per SM / (3 CTAs x 256 threads) = 85, allocated in steps of 8 per thread
        assert regs <= 80, f"{name}: {regs} registers (> 80 leaves two CTAs per SM)"
        assert st == 0 and ld == 0, f"{name}: spills {st}/{ld} bytes"


def _chain_threads():
    src = open(os.path.join(B.CSRC, "gdn_prefill_tc.cu")).read()
    return int(re.search(r"constexpr int kThreads = (\d+);", src).group(1))


def test_chain_kernel_does_not_spill(tmp_path):
    """One CTA per SM: the CTA's warps at the kernel's register count (allocated in steps
    of 8 a thread) must fit the 65,536 registers, with nothing spilled."""
    threads = _chain_threads()
    rep = _ptxas_report("gdn_prefill_tc.cu", tmp_path)
    chain = {k: v for k, v in rep.items() if "prefill_tc_kernel" in k}
    assert chain, sorted(rep)
    for name, (regs, st, ld) in chain.items():
        assert (regs + 7) // 8 * 8 * threads <= 65536, f"{name}: {regs} registers x {threads} threads exceed the SM"
        assert st == 0 and ld == 0, f"{name}: spills {st}/{ld} bytes"
