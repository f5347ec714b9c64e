"""Regenerate the golden fixtures from the reference's own torch implementation.

Runs only where the reference checkout is present (it is not needed, and not
read, by the tests):

    python tests/golden/make_golden.py <path of the reference checkout>

For each case in fixtures.CASES it regenerates the inputs, calls the
reference's ``run`` (``solution/gdn_baseline_torch.py:12-91`` for Hq=16/Hv=32,
``local_test/origina_gdn_prefill.py:20-98`` for Hq=4/Hv=8; decode cases call
``run`` with cu_seqlens = arange(B+1) on [B,H,D] views) and stores the outputs.
"""

from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import fixtures  # noqa: E402


def _load_module(path: str, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main(ref_root: str) -> None:
    run16 = _load_module(os.path.join(ref_root, "solution", "gdn_baseline_torch.py"), "ref16").run
    run4 = _load_module(os.path.join(ref_root, "local_test", "origina_gdn_prefill.py"), "ref4").run
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for name, c in fixtures.CASES.items():
        inp = fixtures.make_inputs(name)
        run = run16 if (c["Hq"], c["Hv"]) == (16, 32) else run4
        if c["kind"] == "prefill":
            out, ns = run(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"],
                          inp["dt_bias"], inp["b"], inp["cu_seqlens"], inp["scale"])
        else:
            B, Hq, Hv = c["B"], c["Hq"], c["Hv"]
            cu = torch.arange(B + 1, dtype=torch.int32)
            out, ns = run(inp["q"].view(B, Hq, -1), inp["k"].view(B, Hq, -1),
                          inp["v"].view(B, Hv, -1), inp["state"], inp["A_log"],
                          inp["a"].view(B, Hv), inp["dt_bias"], inp["b"].view(B, Hv), cu,
                          inp["scale"])
            out = out.unsqueeze(1)
        flat = ns.reshape(-1).numpy()
        idx = fixtures.sample_indices(flat.size, c["sample_stride"])
        np.savez_compressed(
            os.path.join(fixtures.HERE, name + ".npz"),
            out=out.contiguous().view(torch.int16).numpy().view(np.uint16),
            out_shape=np.array(out.shape, dtype=np.int64),
            state_shape=np.array(ns.shape, dtype=np.int64),
            state_idx=idx,
            state_val=flat[idx].astype(np.float32),
            state_sum=ns.double().sum(dim=(-1, -2)).numpy(),
            input_sha=np.array(fixtures.input_sha(inp)),
        )
        print(f"{name}: out {tuple(out.shape)} new_state {tuple(ns.shape)} "
              f"sampled {idx.size} max|state| {float(ns.abs().max()):.4f}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of the reference checkout>")
    main(sys.argv[1])
