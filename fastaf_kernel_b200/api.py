"""Reference-facing entry points: ``kernel`` (varlen prefill) and ``kernel_decode``.

Drop-in for ``solution/triton/kernel.py:416-556`` of the reference: same
positional signatures, same value-returning convention, same output shapes and
dtypes.  Both call hand-written sm_100a CUDA kernels through the C ABI
(include/gdn_b200.h) on the current torch CUDA stream.  There is no CPU path:
inputs must live on a CUDA device and the library must be built.

Additions over the reference, all keyword-only so the positional contract is
unchanged:
  * ``output=`` / ``new_state=`` preallocated destinations (the harness's
    destination-passing style, scripts/replay_first_workload.py:113-116);
  * ``kernel_decode(..., new_state=state)`` updates the state in place;
  * ``method=`` chooses the prefill kernel: "tcgen05" (chunk prep + chain kernels on
    the 5th-generation tensor cores), "chunked" (mma.sync), "recurrent" (CUDA cores)
    or "auto" (what ``prefill_method`` reports);
  * ``use_qk_l2norm=True`` L2-normalises every q and k head vector first,
    x <- bf16(x / sqrt(sum x^2 + 1e-6)) in fp32 -- the normalisation Gated DeltaNet
    layers apply before the recurrence (fused into the decode kernel; a pre-pass for
    prefill).  Off by default: the reference never normalises;
  * ``output_gate=z, norm_weight=w`` (optionally ``norm_eps=``) apply the gated
    RMSNorm of Gated DeltaNet layers to the output,
    o <- o / sqrt(mean(o^2) + eps) * w * silu(z) per head vector (``output_gate``
    below); the reference returns o itself.
"""

from __future__ import annotations

import contextlib
import math
from typing import Callable, Optional, Tuple

import torch

from . import _lib

__all__ = ["kernel", "kernel_decode", "kernel_dps", "kernel_decode_dps", "device_status",
           "prefill_method", "output_gate", "decode_step"]

_GATE_DTYPES = {torch.float32: _lib.GDN_DTYPE_F32, torch.bfloat16: _lib.GDN_DTYPE_BF16}
_METHODS = {"auto": _lib.GDN_PREFILL_AUTO, "chunked": _lib.GDN_PREFILL_CHUNKED,
            "recurrent": _lib.GDN_PREFILL_RECURRENT, "tcgen05": _lib.GDN_PREFILL_TCGEN05}


def prefill_method(total_tokens: int, method: str = "auto", num_seqs: int = 1) -> str:
    """Name of the prefill kernel a call with ``method`` runs for ``total_tokens``
    packed tokens in ``num_seqs`` sequences on the current CUDA device (the C
    library's own choice)."""
    if method not in _METHODS:
        raise ValueError(f"method must be one of {sorted(_METHODS)}")
    code = _lib.load().gdn_prefill_resolve(int(total_tokens), int(num_seqs), _METHODS[method])
    return {v: k for k, v in _METHODS.items()}[code]


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _require_cuda(name: str, t: torch.Tensor, device: torch.device) -> None:
    # (integer device indices: cheaper than building torch.device objects on every call)
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (there is no CPU path), got {t.device}")
    if t.get_device() != device.index:
        raise ValueError(f"{name} is on {t.device}, expected {device}")


def _on_device(device: torch.device):
    """(context making ``device`` current, its current stream's raw handle); the context
    is a no-op when ``device`` is already current (the common case: no device switch)."""
    if device.index == torch.cuda.current_device():
        return contextlib.nullcontext(), torch.cuda.current_stream().cuda_stream
    return torch.cuda.device(device), torch.cuda.current_stream(device).cuda_stream


def _bf16(name: str, t: torch.Tensor) -> torch.Tensor:
    if t.dtype != torch.bfloat16:
        raise TypeError(f"{name} must be bfloat16, got {t.dtype}")
    return t.contiguous()


def _gate(t: torch.Tensor) -> torch.Tensor:
    # a/b and A_log/dt_bias are read as fp32 or bf16; anything else is cast to fp32
    # (the reference upcasts every gate input with .float(), gdn_baseline_torch.py:42-44).
    if t.dtype not in _GATE_DTYPES:
        t = t.float()
    return t.contiguous()


def _gate_rows(t: torch.Tensor, Hv: int) -> Tuple[torch.Tensor, int]:
    """Gate inputs a or b as the kernels read them: rows of Hv elements, element h of row r
    at r * stride + h.  A view whose last dimension is contiguous, in fp32 or bf16 -- such
    as a slice of the projection GEMM's output that holds a and b side by side -- passes as
    it is, with its row stride in elements (0 when packed); anything else becomes a packed
    copy (fp32 unless bf16)."""
    if t.dtype not in _GATE_DTYPES:
        t = t.float()
    lead = [st for n, st in zip(t.shape[:-1], t.stride()[:-1]) if n != 1]
    if t.dim() >= 1 and t.shape[-1] == Hv and (t.stride(-1) == 1 or Hv == 1):
        if not lead:
            return t, 0
        if len(lead) == 1 and lead[0] >= Hv:
            return t, (0 if lead[0] == Hv else int(lead[0]))
    return t.contiguous(), 0


def _scale(scale, D: int) -> float:
    # solution/triton/kernel.py:438-439: a falsy scale selects 1/sqrt(D).
    if not scale or scale == 0.0:
        return 1.0 / math.sqrt(D)
    return float(scale)


def _check_cu_seqlens_host(cu: torch.Tensor, T: int) -> None:
    if cu.numel() < 1:
        raise ValueError("cu_seqlens must have at least one entry")
    if int(cu[0]) != 0 or int(cu[-1]) != T:
        raise ValueError(f"cu_seqlens must start at 0 and end at T={T}, got "
                         f"{int(cu[0])}..{int(cu[-1])}")
    if cu.numel() > 1 and bool((cu[1:] < cu[:-1]).any()):
        raise ValueError("cu_seqlens must be non-decreasing")


def kernel(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, state: Optional[torch.Tensor],
           A_log: torch.Tensor, a: torch.Tensor, dt_bias: torch.Tensor, b: torch.Tensor,
           cu_seqlens: torch.Tensor, scale: Optional[float], *,
           output: Optional[torch.Tensor] = None, new_state: Optional[torch.Tensor] = None,
           method: str = "auto", validate: bool = True,
           use_qk_l2norm: bool = False, output_gate: Optional[torch.Tensor] = None,
           norm_weight: Optional[torch.Tensor] = None,
           norm_eps: float = 1e-6) -> Tuple[torch.Tensor, torch.Tensor]:
    """Varlen Gated DeltaNet prefill (solution/triton/kernel.py:416-489).

    q, k [T, Hq, D] bf16; v [T, Hv, D] bf16; state [N, Hv, D, D] fp32 k-last or
    None; A_log, dt_bias [Hv]; a, b [T, Hv]; cu_seqlens [N+1] (any int dtype;
    cast to int32 as the reference does, :458).  Returns
    (output [T, Hv, D] bf16, new_state [N, Hv, D, D] fp32).

    cu_seqlens must start at 0, end at T and never decrease.  A host (CPU) cu_seqlens
    is checked here when ``validate`` is true (the default); a device-resident one is
    checked by the kernels themselves, so a call never synchronizes with the device to
    check it: the kernels clamp bad entries (no out-of-bounds access) and record the
    error, which ``device_status()`` raises as ValueError.
    """
    device = q.device
    for name, t in (("q", q), ("k", k), ("v", v), ("A_log", A_log), ("a", a),
                    ("dt_bias", dt_bias), ("b", b)):
        _require_cuda(name, t, device)
    if q.dim() != 3 or k.dim() != 3 or v.dim() != 3:
        raise ValueError("q, k, v must be [T, H, D]")
    T, Hq, D = q.shape
    Hv = v.shape[1]
    if k.shape != q.shape:
        raise ValueError(f"k shape {tuple(k.shape)} must equal q shape {tuple(q.shape)}")
    if v.shape[0] != T or v.shape[2] != D:
        raise ValueError(f"v shape {tuple(v.shape)} does not match q {tuple(q.shape)}")
    if a.shape != (T, Hv) or b.shape != (T, Hv):
        raise ValueError(f"a and b must be [T, Hv] = [{T}, {Hv}]")
    if A_log.numel() != Hv or dt_bias.numel() != Hv:
        raise ValueError(f"A_log and dt_bias must have Hv={Hv} elements")
    if cu_seqlens.dim() != 1:
        raise ValueError("cu_seqlens must be 1-D")
    N = cu_seqlens.shape[0] - 1
    if N < 0:
        raise ValueError("cu_seqlens must have at least one entry")
    if validate and not cu_seqlens.is_cuda:
        _check_cu_seqlens_host(cu_seqlens.detach().to(torch.int64), T)
    cu = cu_seqlens.to(device=device, dtype=torch.int32).contiguous()
    scale = _scale(scale, D)

    q, k, v = _bf16("q", q), _bf16("k", k), _bf16("v", v)
    # a and b may be views into a wider projection output (read through their row stride)
    (a, sa), (b, sb) = _gate_rows(a, Hv), _gate_rows(b, Hv)
    A_log, dt_bias = _gate(A_log), _gate(dt_bias)
    if a.dtype != b.dtype:
        b, sb = b.to(a.dtype).contiguous(), 0
    if (sa or sb) and (output_gate is not None or norm_weight is not None):
        (a, sa), (b, sb) = (a.contiguous(), 0), (b.contiguous(), 0)   # the gated entry takes packed gates
    if A_log.dtype != dt_bias.dtype:
        dt_bias = dt_bias.to(A_log.dtype)
    if state is not None:
        _require_cuda("state", state, device)
        if tuple(state.shape) != (N, Hv, D, D):
            raise ValueError(f"state must be [N, Hv, D, D] = [{N}, {Hv}, {D}, {D}]")
        state = state.to(torch.float32).contiguous()
    if output is None:
        output = torch.empty((T, Hv, D), dtype=torch.bfloat16, device=device)
    elif (output.dtype != torch.bfloat16 or tuple(output.shape) != (T, Hv, D)
          or not output.is_contiguous() or output.device != device):
        raise ValueError("output must be a contiguous bf16 [T, Hv, D] tensor on q's device")
    if new_state is None:
        new_state = torch.empty((N, Hv, D, D), dtype=torch.float32, device=device)
    elif (new_state.dtype != torch.float32 or tuple(new_state.shape) != (N, Hv, D, D)
          or not new_state.is_contiguous() or new_state.device != device):
        raise ValueError("new_state must be a contiguous fp32 [N, Hv, D, D] tensor on q's device")
    if method not in _METHODS:
        raise ValueError(f"method must be one of {sorted(_METHODS)}")

    lib = _lib.load()
    ctx, stream = _on_device(device)
    with ctx:
        flags = _lib.GDN_FLAG_QK_L2NORM if use_qk_l2norm else 0
        if output_gate is None and norm_weight is None and (sa or sb):
            _lib.check(lib.gdn_prefill_strided(
                _ptr(q), _ptr(k), _ptr(v), _ptr(state), _ptr(A_log), _ptr(a), _ptr(dt_bias),
                _ptr(b), _ptr(cu), N, T, Hq, Hv, D, scale, _GATE_DTYPES[a.dtype],
                _GATE_DTYPES[A_log.dtype], _ptr(output), _ptr(new_state), sa, sb, _METHODS[method], flags,
                stream))
        elif output_gate is None and norm_weight is None:
            _lib.check(lib.gdn_prefill_flags(
                _ptr(q), _ptr(k), _ptr(v), _ptr(state), _ptr(A_log), _ptr(a), _ptr(dt_bias),
                _ptr(b), _ptr(cu), N, T, Hq, Hv, D, scale, _GATE_DTYPES[a.dtype],
                _GATE_DTYPES[A_log.dtype], _ptr(output), _ptr(new_state), _METHODS[method], flags, stream))
        else:
            z, w = _check_output_gate(output, output_gate, norm_weight, norm_eps)
            _lib.check(lib.gdn_prefill_gated(
                _ptr(q), _ptr(k), _ptr(v), _ptr(state), _ptr(A_log), _ptr(a), _ptr(dt_bias),
                _ptr(b), _ptr(cu), N, T, Hq, Hv, D, scale, _GATE_DTYPES[a.dtype],
                _GATE_DTYPES[A_log.dtype], _ptr(output), _ptr(new_state), _ptr(z), _ptr(w),
                _GATE_DTYPES[w.dtype], float(norm_eps), _METHODS[method], flags, stream))
    return output, new_state


def _prepare_decode(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state):
    """kernel_decode's argument checks and conversions (launches nothing): the tensors the
    kernel reads, the output buffers (allocated when None) and B, Hq, Hv, D, scale."""
    device = q.device
    for name, t in (("q", q), ("k", k), ("v", v), ("A_log", A_log), ("a", a),
                    ("dt_bias", dt_bias), ("b", b)):
        _require_cuda(name, t, device)
    if q.dim() != 4 or q.shape[1] != 1:
        raise ValueError("q must be [B, 1, Hq, D]")
    B, _, Hq, D = q.shape
    Hv = v.shape[2]
    if k.shape != q.shape:
        raise ValueError(f"k shape {tuple(k.shape)} must equal q shape {tuple(q.shape)}")
    if tuple(v.shape) != (B, 1, Hv, D):
        raise ValueError(f"v must be [B, 1, Hv, D], got {tuple(v.shape)}")
    if a.numel() != B * Hv or b.numel() != B * Hv:
        raise ValueError(f"a and b must be [B, 1, Hv] = [{B}, 1, {Hv}]")
    if A_log.numel() != Hv or dt_bias.numel() != Hv:
        raise ValueError(f"A_log and dt_bias must have Hv={Hv} elements")
    scale = _scale(scale, D)
    q, k, v = _bf16("q", q), _bf16("k", k), _bf16("v", v)
    # a and b may be views into a wider projection output (read through their row stride)
    (a, sa), (b, sb) = _gate_rows(a, Hv), _gate_rows(b, Hv)
    A_log, dt_bias = _gate(A_log), _gate(dt_bias)
    if a.dtype != b.dtype:
        b, sb = b.to(a.dtype).contiguous(), 0
    if A_log.dtype != dt_bias.dtype:
        dt_bias = dt_bias.to(A_log.dtype)
    inplace = new_state is not None and state is not None and new_state.data_ptr() == state.data_ptr()
    if state is not None:
        _require_cuda("state", state, device)
        if tuple(state.shape) != (B, Hv, D, D):
            raise ValueError(f"state must be [B, Hv, D, D] = [{B}, {Hv}, {D}, {D}]")
        if inplace:
            if state.dtype != torch.float32 or not state.is_contiguous():
                raise ValueError("in-place decode needs a contiguous fp32 state")
        else:
            state = state.to(torch.float32).contiguous()
    if output is None:
        output = torch.empty((B, 1, Hv, D), dtype=torch.bfloat16, device=device)
    elif (output.dtype != torch.bfloat16 or output.numel() != B * Hv * D
          or not output.is_contiguous() or output.device != device):
        raise ValueError("output must be a contiguous bf16 [B, 1, Hv, D] tensor on q's device")
    if new_state is None:
        new_state = torch.empty((B, Hv, D, D), dtype=torch.float32, device=device)
    elif (new_state.dtype != torch.float32 or tuple(new_state.shape) != (B, Hv, D, D)
          or not new_state.is_contiguous() or new_state.device != device):
        raise ValueError("new_state must be a contiguous fp32 [B, Hv, D, D] tensor on q's device")

    return q, k, v, state, A_log, a, dt_bias, b, output, new_state, B, Hq, Hv, D, scale, sa, sb


def kernel_decode(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                  state: Optional[torch.Tensor], A_log: torch.Tensor, a: torch.Tensor,
                  dt_bias: torch.Tensor, b: torch.Tensor, scale: Optional[float], *,
                  output: Optional[torch.Tensor] = None,
                  new_state: Optional[torch.Tensor] = None,
                  use_qk_l2norm: bool = False, output_gate: Optional[torch.Tensor] = None,
                  norm_weight: Optional[torch.Tensor] = None,
                  norm_eps: float = 1e-6) -> Tuple[torch.Tensor, torch.Tensor]:
    """Single-token Gated DeltaNet decode (solution/triton/kernel.py:492-556).

    q, k [B, 1, Hq, D] bf16; v [B, 1, Hv, D] bf16; a, b [B, 1, Hv];
    state [B, Hv, D, D] fp32 or None.  Returns (output [B, 1, Hv, D] bf16,
    new_state [B, Hv, D, D] fp32).  Pass ``new_state=state`` to update the state
    in place (no second 2 MiB-per-sequence buffer).
    """
    (q, k, v, state, A_log, a, dt_bias, b, output, new_state, B, Hq, Hv, D, scale, sa, sb) = _prepare_decode(
        q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state)
    device = q.device
    lib = _lib.load()
    ctx, stream = _on_device(device)
    with ctx:
        _lib.check(lib.gdn_decode_strided(
            _ptr(q), _ptr(k), _ptr(v), _ptr(state), _ptr(A_log), _ptr(a), _ptr(dt_bias),
            _ptr(b), B, Hq, Hv, D, scale, _GATE_DTYPES[a.dtype], _GATE_DTYPES[A_log.dtype],
            _ptr(output), _ptr(new_state), sa, sb, _lib.GDN_FLAG_QK_L2NORM if use_qk_l2norm else 0,
            stream))
    if output_gate is not None or norm_weight is not None:
        _gated_rmsnorm(output, output_gate, norm_weight, norm_eps)
    return output, new_state


def output_gate(output: torch.Tensor, gate: torch.Tensor, weight: torch.Tensor,
                eps: float = 1e-6) -> torch.Tensor:
    """In place: output <- output / sqrt(mean(output^2) + eps) * weight * silu(gate) over
    every 128-element head vector (the gated RMSNorm Gated DeltaNet layers apply before
    the output projection).  output, gate: bf16 of the same shape [..., D] on one CUDA
    device; weight [D] fp32 or bf16.  Returns ``output``."""
    return _gated_rmsnorm(output, gate, weight, eps)


def _check_output_gate(output, gate, weight, eps):
    """Validated (gate bf16 contiguous, weight fp32/bf16 contiguous) for gating ``output``."""
    if gate is None or weight is None:
        raise ValueError("output gating needs both a gate and a norm weight")
    if not eps >= 0.0:
        raise ValueError("eps must be >= 0")
    device = output.device
    _require_cuda("output", output, device)
    _require_cuda("gate", gate, device)
    _require_cuda("weight", weight, device)
    if output.dtype != torch.bfloat16 or not output.is_contiguous():
        raise ValueError("output must be a contiguous bf16 tensor")
    if tuple(gate.shape) != tuple(output.shape):
        raise ValueError(f"gate shape {tuple(gate.shape)} must equal output shape {tuple(output.shape)}")
    D = output.shape[-1]
    if weight.numel() != D:
        raise ValueError(f"weight must have {D} elements")
    return _bf16("gate", gate), _gate(weight)


def _gated_rmsnorm(output, gate, weight, eps):
    gate, weight = _check_output_gate(output, gate, weight, eps)
    device = output.device
    D = output.shape[-1]
    lib = _lib.load()
    ctx, stream = _on_device(device)
    with ctx:
        _lib.check(lib.gdn_output_gate(_ptr(output), _ptr(gate), _ptr(weight), _GATE_DTYPES[weight.dtype],
                                       output.numel() // D, D, float(eps), stream))
    return output


def decode_step(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, state: torch.Tensor,
                A_log: torch.Tensor, a: torch.Tensor, dt_bias: torch.Tensor, b: torch.Tensor,
                scale: Optional[float], output: torch.Tensor, new_state: torch.Tensor, *,
                use_qk_l2norm: bool = False) -> Callable[[], None]:
    """A prepared decode step over fixed buffers, for serving loops that refill q, k, v,
    a and b in place every token: the arguments are checked once, here, exactly as by
    ``kernel_decode``; each call of the returned function then only launches the step on
    the device's current stream (about 5 us of host time, against about 17 us for a
    ``kernel_decode`` call that re-checks everything).  The buffers must stay alive and
    keep their storage (no resize or ``set_``) while the step is used; ``new_state`` may
    be ``state`` (in place).  No output gating here (use ``output_gate`` after it)."""
    if output is None or new_state is None or state is None:
        raise ValueError("decode_step needs its state, output and new_state buffers")
    given = (q, k, v, state, A_log, a, dt_bias, b)
    prep = _prepare_decode(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state)
    # the step keeps the buffers' addresses, so none of them may have needed a converted copy
    for name, t, u in zip(("q", "k", "v", "state", "A_log", "a", "dt_bias", "b"), given, prep[:8]):
        if u.data_ptr() != t.data_ptr():
            raise ValueError(f"decode_step needs {name} contiguous in a dtype the kernel reads directly "
                             "(with a and b of one dtype, A_log and dt_bias of one dtype)")
    q, k, v, state, A_log, a, dt_bias, b, output, new_state, B, Hq, Hv, D, scale, sa, sb = prep
    device = q.device
    lib = _lib.load()
    fn = lib.gdn_decode_strided
    head = (_ptr(q), _ptr(k), _ptr(v), _ptr(state), _ptr(A_log), _ptr(a), _ptr(dt_bias), _ptr(b), B, Hq, Hv, D,
            scale, _GATE_DTYPES[a.dtype], _GATE_DTYPES[A_log.dtype], _ptr(output), _ptr(new_state), sa, sb,
            _lib.GDN_FLAG_QK_L2NORM if use_qk_l2norm else 0)
    index = device.index
    # the raw handle of a device's current stream without building a Stream object
    # (torch's own fast getter where this torch has it)
    raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    current = (lambda: raw(index)) if raw is not None else (lambda: torch.cuda.current_stream(index).cuda_stream)

    def step() -> None:
        if torch.cuda.current_device() == index:
            rc = fn(*head, current())
        else:
            with torch.cuda.device(index):
                rc = fn(*head, current())
        if rc != 0:
            _lib.check(rc)
    return step


def kernel_dps(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output, new_state):
    """Destination-passing prefill: ``runnable(*inputs, *outputs)``
    (scripts/replay_first_workload.py:113-116)."""
    kernel(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale,
           output=output, new_state=new_state)


def kernel_decode_dps(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state):
    """Destination-passing decode; ``new_state`` may be ``state`` (in place)."""
    kernel_decode(q, k, v, state, A_log, a, dt_bias, b, scale, output=output,
                  new_state=new_state)


def device_status(device: Optional[torch.device] = None) -> None:
    """Synchronize the current stream and raise what the kernels recorded on the device
    since the last check (the record is then cleared): ``GdnError`` (status
    GDN_ERR_DEVICE_TIMEOUT) if a tcgen05 prefill CTA gave up on a bounded device-side
    wait, ``ValueError`` if a prefill read a malformed device-resident cu_seqlens."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    with torch.cuda.device(device):
        _lib.check(_lib.load().gdn_device_status(torch.cuda.current_stream(device).cuda_stream))
