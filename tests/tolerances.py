"""Parity tolerances of the Gated DeltaNet kernels against the CPU oracle.

output    : |got - ref| <= ATOL + RTOL * |ref| elementwise (bf16 outputs)
new_state : max|got - ref| / max|ref| <= STATE_MAX_REL (fp32 state)

Max relative error is taken against the largest reference magnitude, since an
elementwise ratio is unbounded where the reference is near zero.
"""
import torch

ATOL = 2e-2
RTOL = 2e-2
STATE_MAX_REL = 1e-3


def state_max_rel(got: torch.Tensor, ref: torch.Tensor) -> float:
    got = got.detach().double().cpu()
    ref = ref.detach().double().cpu()
    denom = ref.abs().max().item()
    diff = (got - ref).abs().max().item()
    return diff / denom if denom > 0 else diff


def output_excess(got: torch.Tensor, ref: torch.Tensor, atol=ATOL, rtol=RTOL) -> float:
    """max(|got-ref| - (atol + rtol*|ref|)); <= 0 means within tolerance."""
    got = got.detach().float().cpu()
    ref = ref.detach().float().cpu()
    if got.numel() == 0:
        return -1.0
    return ((got - ref).abs() - (atol + rtol * ref.abs())).max().item()


def assert_parity(out, ref_out, ns, ref_ns, state_tol=STATE_MAX_REL, atol=ATOL, rtol=RTOL):
    assert out.shape == ref_out.shape, (out.shape, ref_out.shape)
    assert ns.shape == ref_ns.shape, (ns.shape, ref_ns.shape)
    assert torch.isfinite(out.float()).all(), "non-finite output"
    assert torch.isfinite(ns).all(), "non-finite new_state"
    ex = output_excess(out, ref_out, atol, rtol)
    assert ex <= 0, f"output exceeds atol={atol}/rtol={rtol} by {ex:.3e}"
    rel = state_max_rel(ns, ref_ns)
    assert rel <= state_tol, f"new_state max rel error {rel:.3e} > {state_tol:.1e}"
    return ex, rel
