"""The reference's own Triton GPU kernels, compiled ahead of time for B200 (sm_100):
measurement infrastructure, not part of the library (nothing in fastaf_kernel_b200/
imports it).

The reference's GPU path is two Triton kernels, each autotuned over a list of launch
configurations (solution/triton/kernel.py:36-106):
  * _gdn_prefill_kernel_v2 (solution/triton/kernel.py:138-278), launched by `kernel`
    (:416-489) on a grid (D / BLOCK_V, N, Hv);
  * _gdn_decode_kernel_v3 (:285-409), launched by `kernel_decode` (:492-556) on a grid
    (D / BLOCK_V, B, Hv).

`build(reference_root)` runs in the container that holds the reference checkout.  It
compiles every configuration of both lists from the reference's sources where they lie,
for the shapes bench.py times (the 16 x 8192 prefill with Hq 16 / Hv 32 and an initial
state, and the B = 512 decode with a state), with the specialisations Triton's JIT picks
for those calls.  It keeps only the compiled cubins and their metadata under oracle/_ref/
(git-ignored): no reference source, and no intermediate representation, travels.

`RefTriton` reloads them on the GPU box through Triton's own runtime (CompiledKernel and
the launcher Triton generates).  It autotunes the way the reference's autotuner does,
taking the fastest configuration of the list on the same inputs, and launches with the
reference entry points' argument conventions.
"""

from __future__ import annotations

import glob
import json
import math
import os
import shutil
import tempfile
from types import SimpleNamespace
from typing import Dict, List, Optional

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref", "triton")
# Where the reference checkout lives in the build container (absent on the GPU box, which
# only loads what build() wrote).
REFERENCE_ROOT = os.environ.get("GDN_REFERENCE_ROOT", "/root/reference")

# The shapes the compiled specialisations are for (bench.py's workloads).
PREFILL_SHAPE = dict(T=16 * 8192, N=16, Hq=16, Hv=32, D=128)
DECODE_SHAPE = dict(B=512, Hq=16, Hv=32, D=128)


def _prefill_args(q, k, v, state_in, new_state, A_log, a, dt_bias, b, cu, out, scale, gv_ratio):
    """The non-keyword arguments of `kernel`'s launch (solution/triton/kernel.py:466-485)."""
    return (q, k, v, A_log, a, dt_bias, b, state_in, new_state, out, cu,
            q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2),
            v.stride(0), v.stride(1), v.stride(2), a.stride(0), a.stride(1), b.stride(0), b.stride(1),
            new_state.stride(0), new_state.stride(1), new_state.stride(2), new_state.stride(3),
            out.stride(0), out.stride(1), out.stride(2), gv_ratio, float(scale))


def _decode_args(q, k, v, state_in, new_state, A_log, a, dt_bias, b, out, scale, gv_ratio):
    """The non-keyword arguments of `kernel_decode`'s launch (solution/triton/kernel.py:535-551);
    q, k, v, a, b, out already squeezed to [B, H, ...]."""
    return (q, k, v, A_log, a, dt_bias, b, state_in, new_state, out,
            q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2),
            v.stride(0), v.stride(1), v.stride(2), a.stride(0), a.stride(1), b.stride(0), b.stride(1),
            new_state.stride(0), new_state.stride(1), new_state.stride(2), new_state.stride(3),
            out.stride(0), out.stride(1), out.stride(2), gv_ratio, float(scale))


def build(reference_root: str, out_dir: str = OUT_DIR) -> int:
    """Compile every configuration of both kernels for sm_100; returns how many were
    written (0 when the reference checkout is absent)."""
    path = os.path.join(reference_root, "solution", "triton", "kernel.py")
    if not os.path.exists(path):
        return 0
    import importlib.util

    import torch
    import triton
    from triton.backends.compiler import GPUTarget
    from triton.runtime import driver

    class _TargetOnly:
        """Stands in for the CUDA driver while compiling (no GPU here): it only names the
        target, so Triton compiles without touching a device."""

        def get_current_device(self):
            return 0

        def get_current_stream(self, device=None):
            return 0

        def get_current_target(self):
            return GPUTarget("cuda", 100, 32)

        def get_active_torch_device(self):
            return torch.device("cpu")

    cache = tempfile.mkdtemp(prefix="gdn_ref_triton_")
    old_cache = triton.knobs.cache.dir
    triton.knobs.cache.dir = cache
    old_active = driver._active     # (None until a real driver was first used)
    driver.set_active(_TargetOnly())
    written = 0
    try:
        spec = importlib.util.spec_from_file_location("gdn_reference_triton_kernel", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        if os.path.isdir(out_dir):
            shutil.rmtree(out_dir)
        os.makedirs(out_dir)
        P, Dd = PREFILL_SHAPE, DECODE_SHAPE
        bf, f32 = torch.bfloat16, torch.float32
        # CPU stand-ins with the shapes and strides of the timed calls (Triton specialises
        # on strides equal to 1 and on divisibility by 16; every device pointer is aligned)
        q = torch.empty(P["T"], P["Hq"], P["D"], dtype=bf)
        v = torch.empty(P["T"], P["Hv"], P["D"], dtype=bf)
        gates = torch.empty(P["T"], P["Hv"], dtype=bf)
        par = torch.empty(P["Hv"], dtype=f32)
        st = torch.empty(P["N"], P["Hv"], P["D"], P["D"], dtype=f32)
        cu = torch.zeros(P["N"] + 1, dtype=torch.int32)
        pre_args = _prefill_args(q, q, v, st, st, par, gates, par, gates, cu, v, 0.0884,
                                 P["Hv"] // P["Hq"])
        dq = torch.empty(Dd["B"], Dd["Hq"], Dd["D"], dtype=bf)
        dv = torch.empty(Dd["B"], Dd["Hv"], Dd["D"], dtype=bf)
        dg = torch.empty(Dd["B"], Dd["Hv"], dtype=bf)
        dst = torch.empty(Dd["B"], Dd["Hv"], Dd["D"], Dd["D"], dtype=f32)
        dec_args = _decode_args(dq, dq, dv, dst, dst, par, dg, par, dg, dv, 0.0884,
                                Dd["Hv"] // Dd["Hq"])
        for kind, tuned, args in (("prefill", mod._gdn_prefill_kernel_v2, pre_args),
                                  ("decode", mod._gdn_decode_kernel_v3, dec_args)):
            for ci, cfg in enumerate(tuned.configs):
                ck = tuned.fn.warmup(*args, grid=(1,), HAS_STATE=1, HEAD_SIZE=128, **cfg.kwargs,
                                     num_warps=cfg.num_warps, num_stages=cfg.num_stages)
                tag = f"{kind}_{ci:02d}"
                with open(os.path.join(out_dir, tag + ".cubin"), "wb") as f:
                    f.write(ck.asm["cubin"])
                meta_json = next(p for name, p in ck.metadata_group.items() if name.endswith(".json"))
                shutil.copyfile(meta_json, os.path.join(out_dir, tag + ".json"))
                launch = {"kind": kind, "config": cfg.kwargs, "num_warps": cfg.num_warps,
                          "num_stages": cfg.num_stages, "hash": ck.hash,
                          "signature": dict(ck.src.signature),
                          "constants": [[list(k), v] for k, v in ck.src.constants.items()]}
                with open(os.path.join(out_dir, tag + ".launch.json"), "w") as f:
                    json.dump(launch, f)
                written += 1
    finally:
        driver._active = old_active
        triton.knobs.cache.dir = old_cache
        shutil.rmtree(cache, ignore_errors=True)   # the cache's source and IR copies go with it
    return written


def available(out_dir: str = OUT_DIR) -> bool:
    return bool(glob.glob(os.path.join(out_dir, "*.launch.json")))


def build_if_stale(reference_root: str = REFERENCE_ROOT, out_dir: str = OUT_DIR) -> int:
    """build() unless the compiled kernels are newer than the reference's kernel file and
    this recipe; returns the number of compiled configurations present."""
    path = os.path.join(reference_root, "solution", "triton", "kernel.py")
    specs = glob.glob(os.path.join(out_dir, "*.launch.json"))
    if not os.path.exists(path):
        return len(specs)
    newest_input = max(os.path.getmtime(path), os.path.getmtime(os.path.abspath(__file__)))
    if specs and min(os.path.getmtime(p) for p in specs) > newest_input:
        return len(specs)
    return build(reference_root, out_dir)


class RefTriton:
    """The compiled reference kernels on the current CUDA device."""

    def __init__(self, out_dir: str = OUT_DIR):
        from triton.compiler.compiler import CompiledKernel
        self.kernels: Dict[str, List[tuple]] = {"prefill": [], "decode": []}
        for spec_path in sorted(glob.glob(os.path.join(out_dir, "*.launch.json"))):
            tag = os.path.basename(spec_path)[:-len(".launch.json")]
            with open(spec_path) as f:
                s = json.load(f)
            src = SimpleNamespace(signature=s["signature"],
                                  constants={tuple(k): v for k, v in s["constants"]})
            group = {tag + ".json": os.path.join(out_dir, tag + ".json"),
                     tag + ".cubin": os.path.join(out_dir, tag + ".cubin")}
            self.kernels[s["kind"]].append((CompiledKernel(src, group, s["hash"]), s))
        if not self.kernels["prefill"] or not self.kernels["decode"]:
            raise RuntimeError(f"no compiled reference kernels under {out_dir}")
        self.best: Dict[str, Optional[int]] = {"prefill": None, "decode": None}
        self.tried: Dict[str, int] = {"prefill": 0, "decode": 0}

    @staticmethod
    def _launch(ck, s, grid, args):
        """Launch with every parameter in order: the runtime arguments and strides, then
        the keyword compile-time ones (HAS_STATE, HEAD_SIZE, BLOCK_V[, BLOCK_K]).  Triton's
        launcher skips the compile-time values; the strides it specialised to a constant
        must equal the ones passed."""
        cfg = s["config"]
        full = list(args) + [1, 128, cfg["BLOCK_V"]] + ([cfg["BLOCK_K"]] if s["kind"] == "decode" else [])
        if len(full) != len(s["signature"]):
            raise RuntimeError(f"{len(full)} arguments for a {len(s['signature'])}-parameter kernel")
        for (i,), v in ((tuple(k), v) for k, v in s["constants"]):
            if full[i] != v:
                raise RuntimeError(f"argument {list(s['signature'])[i]} = {full[i]}, compiled for {v}")
        ck[grid](*full)

    def _autotune(self, kind, rows, Hv, args):
        """The fastest configuration of the list on these inputs (one warm-up and two timed
        launches each, CUDA events), as the reference's autotuner would choose."""
        import torch
        best, best_ms = None, math.inf
        for i, (ck, s) in enumerate(self.kernels[kind]):
            grid = (128 // s["config"]["BLOCK_V"], rows, Hv)
            try:
                self._launch(ck, s, grid, args)
                torch.cuda.synchronize()
            except Exception:       # out of resources for this configuration: pruned
                continue
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(2):
                self._launch(ck, s, grid, args)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / 2
            self.tried[kind] += 1
            if ms < best_ms:
                best, best_ms = i, ms
        if best is None:
            raise RuntimeError(f"no {kind} configuration could be launched")
        self.best[kind] = best
        return best

    def prefill(self, q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output, new_state):
        """`kernel(...)` of the reference with the outputs passed in; state must be given."""
        T, Hq, D = q.shape
        Hv = v.shape[1]
        N = cu_seqlens.shape[0] - 1
        if not scale:
            scale = 1.0 / math.sqrt(D)
        args = _prefill_args(q, k, v, state, new_state, A_log, a, dt_bias, b, cu_seqlens, output,
                             scale, Hv // Hq)
        if self.best["prefill"] is None:
            self._autotune("prefill", N, Hv, args)
        ck, s = self.kernels["prefill"][self.best["prefill"]]
        self._launch(ck, s, (128 // s["config"]["BLOCK_V"], N, Hv), args)

    def decode(self, q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state):
        """`kernel_decode(...)` of the reference with the outputs passed in ([B, 1, H, D]
        inputs, output [B, Hv, D]); state must be given."""
        B, _, Hq, D = q.shape
        Hv = v.shape[2]
        if not scale:
            scale = 1.0 / math.sqrt(D)
        args = _decode_args(q.view(B, Hq, D), k.view(B, Hq, D), v.view(B, Hv, D), state, new_state,
                            A_log, a.view(B, Hv), dt_bias, b.view(B, Hv), output, scale, Hv // Hq)
        if self.best["decode"] is None:
            self._autotune("decode", B, Hv, args)
        ck, s = self.kernels["decode"][self.best["decode"]]
        self._launch(ck, s, (128 // s["config"]["BLOCK_V"], B, Hv), args)

    def config(self, kind):
        i = self.best[kind]
        if i is None:
            return None
        _, s = self.kernels[kind][i]
        return dict(s["config"], num_warps=s["num_warps"], num_stages=s["num_stages"])
