"""Small, self-contained launches of each kernel for profiling under ncu (the
reproducer of the summaries under profiles/; not part of the library).

    python tests/profile_cases.py prefill --seq-len 4096 [--method tcgen05]
    python tests/profile_cases.py decode --batch 512

Each case builds its seeded inputs on cuda:0, runs the kernel a few times (so a
profiler can skip the first launch with `-s`) and exits 0.  Inputs are sized
above the 126 MB L2 but stay a few GB on the device, so a `--set full` capture of
one launch ends in seconds.
"""

from __future__ import annotations

import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from fastaf_kernel_b200 import api  # noqa: E402
from fastaf_kernel_b200 import workloads as W  # noqa: E402


def prefill(seq_len: int, n_seqs: int, method: str, launches: int) -> None:
    dev = torch.device("cuda", 0)
    x = W.prefill_long(seed=3, device=dev, n_seqs=n_seqs, seq_len=seq_len)
    for _ in range(launches):
        api.kernel(x["q"], x["k"], x["v"], x["state"], x["A_log"], x["a"], x["dt_bias"],
                   x["b"], x["cu_seqlens"], x["scale"], method=method, validate=False)
    torch.cuda.synchronize()


def decode(batch: int, launches: int) -> None:
    dev = torch.device("cuda", 0)
    d = {k: (v.to(dev) if isinstance(v, torch.Tensor) else v)
         for k, v in W.decode_inputs(batch, seed=2).items()}
    for _ in range(launches):
        api.kernel_decode(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"],
                          d["b"], d["scale"], new_state=d["state"])
    torch.cuda.synchronize()


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="case", required=True)
    p = sub.add_parser("prefill")
    p.add_argument("--seq-len", type=int, default=4096)
    p.add_argument("--n-seqs", type=int, default=16)
    p.add_argument("--method", choices=["auto", "tcgen05", "chunked", "recurrent"], default="tcgen05")
    p.add_argument("--launches", type=int, default=2)
    d = sub.add_parser("decode")
    d.add_argument("--batch", type=int, default=512)
    d.add_argument("--launches", type=int, default=3)
    args = ap.parse_args(argv)
    if args.case == "prefill":
        prefill(args.seq_len, args.n_seqs, args.method, args.launches)
    else:
        decode(args.batch, args.launches)
    print("ok")
    return 0


if __name__ == "__main__":
    sys.exit(main())
