"""PyTorch custom ops over the C ABI (``torch.ops.svdq_b200.*``).

Each op validates its tensors, allocates outputs with the caching allocator
and calls the corresponding ``extern "C"`` entry point of ``libsvdq_b200.so``
on the caller's current CUDA stream.  CPU tensors are rejected: there is no
CPU implementation behind these ops.
"""
from __future__ import annotations

import collections
import ctypes
import threading
import types
from typing import Optional

import torch

from . import _lib

Tensor = torch.Tensor


def _p(t: Optional[Tensor]):
    return ctypes.c_void_p(t.data_ptr()) if t is not None and t.numel() > 0 else None


def _raw_stream(dev: torch.device) -> int:
    """The current CUDA stream of ``dev`` as a handle (the allocator's fast path, used by every
    call; ``torch.cuda.current_stream`` builds a Python stream object each time)."""
    get = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    if get is not None:
        return int(get(dev.index if dev.index is not None else torch.cuda.current_device()))
    return torch.cuda.current_stream(dev).cuda_stream


def _stream(dev: torch.device):
    return ctypes.c_void_p(_raw_stream(dev))


def _need_cuda(name: str, *ts: Optional[Tensor]) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError(f"svdq_b200.{name}: all tensors must be CUDA tensors (got {t.device}); "
                             "this runtime has no CPU path")


def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def round_up(v: int, m: int) -> int:
    return (v + m - 1) // m * m


def lowrank_width(r_tot: int) -> int:
    """R2: width of the hi/lo low-rank operand (0 when there is no low-rank term)."""
    return round_up(2 * r_tot, 64) if r_tot > 0 else 0


_DT = {torch.bfloat16: _lib.SVDQ_BF16, torch.float16: _lib.SVDQ_FP16, torch.float32: _lib.SVDQ_FP32}


_EAGER: dict = {}


def _op(name: str):
    """Registers the decorated function as the custom op ``svdq_b200::<name>`` and keeps the plain
    function in ``eager`` as well: the module layer calls it directly outside ``torch.compile``,
    which saves the dispatcher's 10-20 us per call (host time that a small layer cannot hide)."""
    def deco(fn):
        _EAGER[name] = fn
        return torch.library.custom_op(f"svdq_b200::{name}", fn, mutates_args=())
    return deco


# --------------------------------------------------------------------------- activation passes
def _lowrank_args(l2, lora_down):
    rank = 0 if l2 is None else l2.shape[0]
    lrank = 0 if lora_down is None else lora_down.shape[0]
    return rank, lrank, lowrank_width(rank + lrank)


_GEMM_WS_KEEP = 8  # workspaces kept per kind (most recently used (device, stream) pairs)
_act_ws: "collections.OrderedDict[tuple, Tensor]" = collections.OrderedDict()
_act_ws_lock = threading.Lock()


def _workspace(m: int, k_pad: int, rank: int, lrank: int, dev: torch.device) -> Tensor:
    """The activation pass's workspace: the fp32 K-slice partials of the low-rank products, which
    every launch writes in full before its finalize launch adds them (no clearing between calls).
    One per (device, stream), kept and grown as larger calls need; launches on one stream run in
    order, so they share it.  Inside a CUDA graph capture a fresh workspace is made, so a graph
    never holds the address of a cached workspace that may be freed later."""
    n = int(_lib.lib().svdq_act_quant_workspace_bytes(m, k_pad, rank, lrank))
    if torch.cuda.is_current_stream_capturing():
        return torch.zeros((max(n, 0),), dtype=torch.uint8, device=dev)
    key = (dev.index, _raw_stream(dev))
    with _act_ws_lock:
        ws = _act_ws.get(key)
        if ws is None or ws.numel() < n:
            ws = torch.zeros((max(n, 2 * (0 if ws is None else ws.numel())),), dtype=torch.uint8, device=dev)
            _act_ws[key] = ws
        _act_ws.move_to_end(key)
        while len(_act_ws) > _GEMM_WS_KEEP:
            _act_ws.popitem(last=False)
    return ws


@_op("act_quant")
def act_quant(x: Tensor, smooth: Tensor, l2: Optional[Tensor], lora_down: Optional[Tensor],
              lora_col_scale: Optional[Tensor], k_pad: int, a_group: int, emit_a16: bool,
              emit_packed: bool) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """W4A4 activation pass: smoothing, dynamic INT4 quantization, low-rank down-projection.

    Returns ``(a16 [M,K_pad] fp16, mid_hl [M,R2] bf16, packed [M,K_pad/2] u8,
    scales [M,K_pad/a_group] bf16)``; outputs that were not requested are empty.
    ``packed``/``scales`` are bit-exact with ``pack_int4(quantize_symmetric_int4(x / smooth,
    a_group))`` of the reference; ``a16`` holds ``q * scale`` exactly.
    """
    _need_cuda("act_quant", x, smooth, l2, lora_down, lora_col_scale)
    _need(x.dim() == 2 and x.dtype == torch.bfloat16, "act_quant: x must be a 2-D bf16 tensor")
    _need(x.stride(1) == 1, "act_quant: x must have unit column stride")
    m, k_in = x.shape
    rank, lrank, r2 = _lowrank_args(l2, lora_down)
    dev = x.device
    a16 = torch.empty((m, k_pad) if emit_a16 else (0,), dtype=torch.float16, device=dev)
    mid = torch.empty((m, r2) if (emit_a16 and r2) else (0,), dtype=torch.bfloat16, device=dev)
    packed = torch.empty((m, k_pad // 2) if emit_packed else (0,), dtype=torch.uint8, device=dev)
    scales = torch.empty((m, k_pad // a_group) if emit_packed else (0,), dtype=torch.bfloat16, device=dev)
    if m == 0:
        return a16, mid, packed, scales
    ws = _workspace(m, k_pad, rank, lrank, dev) if mid.numel() else None
    _lib.call("svdq_act_quant", _p(x), x.stride(0), _p(smooth), _p(l2), rank, _p(lora_down),
              _p(lora_col_scale), lrank, m, k_in, k_pad, a_group, _p(packed), _p(scales), _p(a16),
              _p(mid), r2, _p(ws), 0 if ws is None else ws.numel(), _stream(dev))
    return a16, mid, packed, scales


@act_quant.register_fake
def _(x, smooth, l2, lora_down, lora_col_scale, k_pad, a_group, emit_a16, emit_packed):
    m = x.shape[0]
    _, _, r2 = _lowrank_args(l2, lora_down)
    e = x.new_empty
    return (e((m, k_pad) if emit_a16 else (0,), dtype=torch.float16),
            e((m, r2) if (emit_a16 and r2) else (0,), dtype=torch.bfloat16),
            e((m, k_pad // 2) if emit_packed else (0,), dtype=torch.uint8),
            e((m, k_pad // a_group) if emit_packed else (0,), dtype=torch.bfloat16))


def ascales_ld(m: int) -> int:
    """Row stride of the group-major activation scales of ``act_quant_i8``: M rounded up to 64 (the
    int8 GEMM reads whole 64-token tiles; entries past M are zero)."""
    return round_up(max(m, 1), 64)


@_op("act_quant_i8")
def act_quant_i8(x: Tensor, smooth: Tensor, l2: Optional[Tensor], lora_down: Optional[Tensor],
                 lora_col_scale: Optional[Tensor], k_pad: int, a_group: int) -> tuple[Tensor, Tensor, Tensor]:
    """W4A4 activation pass for the int8-code GEMM: the codes of ``quantize_symmetric_int4(x / smooth,
    a_group)`` as int8 ``[M, K_pad]``, its bf16 scales as fp32 group-major ``[K_pad/a_group,
    ascales_ld(M)]`` (zero past M), and ``mid_hl [M, R2]``."""
    _need_cuda("act_quant_i8", x, smooth, l2, lora_down, lora_col_scale)
    _need(x.dim() == 2 and x.dtype == torch.bfloat16, "act_quant_i8: x must be a 2-D bf16 tensor")
    _need(x.stride(1) == 1, "act_quant_i8: x must have unit column stride")
    m, k_in = x.shape
    rank, lrank, r2 = _lowrank_args(l2, lora_down)
    dev = x.device
    codes = torch.empty((m, k_pad), dtype=torch.int8, device=dev)
    lda = ascales_ld(m)
    ascales = torch.empty((k_pad // a_group, lda), dtype=torch.float32, device=dev)  # the kernel zeroes rows >= M
    mid = torch.empty((m, r2) if r2 else (0,), dtype=torch.bfloat16, device=dev)
    if m == 0:
        return codes, ascales, mid
    ws = _workspace(m, k_pad, rank, lrank, dev) if r2 else None
    _lib.call("svdq_act_quant_i8", _p(x), x.stride(0), _p(smooth), _p(l2), rank, _p(lora_down),
              _p(lora_col_scale), lrank, m, k_in, k_pad, a_group, _p(codes), _p(ascales), lda,
              _p(mid), r2, _p(ws), 0 if ws is None else ws.numel(), _stream(dev))
    return codes, ascales, mid


@act_quant_i8.register_fake
def _(x, smooth, l2, lora_down, lora_col_scale, k_pad, a_group):
    m = x.shape[0]
    _, _, r2 = _lowrank_args(l2, lora_down)
    return (x.new_empty((m, k_pad), dtype=torch.int8),
            x.new_empty((k_pad // a_group, ascales_ld(m)), dtype=torch.float32),
            x.new_empty((m, r2) if r2 else (0,), dtype=torch.bfloat16))


@_op("w4a16_prep")
def w4a16_prep(x: Tensor, smooth: Tensor, l2: Optional[Tensor], lora_down: Optional[Tensor],
               lora_col_scale: Optional[Tensor], k_pad: int) -> tuple[Tensor, Tensor]:
    """W4A16 activation pass: ``a16 = fp16(x / smooth)`` (fp32 division) and the low-rank
    down-projection.  ``l2`` is the fp16 copy of the checkpoint's l2 (made once at load).
    Returns ``(a16 [M,K_pad] fp16, mid_hl [M,R2] bf16)``."""
    _need_cuda("w4a16_prep", x, smooth, l2, lora_down, lora_col_scale)
    _need(x.dim() == 2 and x.dtype == torch.bfloat16, "w4a16_prep: x must be a 2-D bf16 tensor")
    _need(l2 is None or l2.dtype == torch.float16, "w4a16_prep: l2 must be fp16 (convert once at load)")
    _need(x.stride(1) == 1, "w4a16_prep: x must have unit column stride")
    m, k_in = x.shape
    rank, lrank, r2 = _lowrank_args(l2, lora_down)
    a16 = torch.empty((m, k_pad), dtype=torch.float16, device=x.device)
    mid = torch.empty((m, r2) if r2 else (0,), dtype=torch.bfloat16, device=x.device)
    if m == 0:
        return a16, mid
    ws = _workspace(m, k_pad, rank, lrank, x.device) if r2 else None
    _lib.call("svdq_w4a16_prep", _p(x), x.stride(0), _p(smooth), _p(l2), rank, _p(lora_down),
              _p(lora_col_scale), lrank, m, k_in, k_pad, _p(a16), _p(mid), r2, _p(ws),
              0 if ws is None else ws.numel(), _stream(x.device))
    return a16, mid


@w4a16_prep.register_fake
def _(x, smooth, l2, lora_down, lora_col_scale, k_pad):
    m = x.shape[0]
    _, _, r2 = _lowrank_args(l2, lora_down)
    return (x.new_empty((m, k_pad), dtype=torch.float16),
            x.new_empty((m, r2) if r2 else (0,), dtype=torch.bfloat16))


# --------------------------------------------------------------------------- converter
@_op("quantize_weight")
def quantize_weight(w: Tensor, group: int, scale_dtype: torch.dtype) -> tuple[Tensor, Tensor]:
    """fp32 residual ``w [N, K]`` -> ``(packed [N, K_pad/2] u8, scales [N, K_pad/group])``, bit-exact with
    the reference's ``pack_int4(quantize_symmetric_int4(w, group, dim=1))`` (scales rounded once to
    ``scale_dtype``)."""
    _need_cuda("quantize_weight", w)
    _need(w.dim() == 2 and w.dtype == torch.float32 and w.stride(1) == 1, "quantize_weight: w must be fp32 [N, K]")
    _need(scale_dtype in _DT, "quantize_weight: scale_dtype must be float32, float16 or bfloat16")
    n, k = w.shape
    k_pad = round_up(k, group)
    packed = torch.empty((n, k_pad // 2), dtype=torch.uint8, device=w.device)
    scales = torch.empty((n, k_pad // group), dtype=scale_dtype, device=w.device)
    _lib.call("svdq_quantize_weight", _p(w), w.stride(0), n, k, group, _p(packed), _p(scales), _DT[scale_dtype],
              _stream(w.device))
    return packed, scales


@quantize_weight.register_fake
def _(w, group, scale_dtype):
    n, k = w.shape
    k_pad = round_up(k, group)
    return (w.new_empty((n, k_pad // 2), dtype=torch.uint8), w.new_empty((n, k_pad // group), dtype=scale_dtype))


# --------------------------------------------------------------------------- load-time operands
@_op("repack_weight")
def repack_weight(qweight: Tensor, scales: Tensor, w_group: int) -> Tensor:
    """Checkpoint INT4 weight -> ``w16 [N, K_pad]`` fp16 = q * scale."""
    _need_cuda("repack_weight", qweight, scales)
    _need(qweight.dtype == torch.uint8 and qweight.dim() == 2 and qweight.is_contiguous(),
          "repack_weight: qweight must be contiguous uint8 [N, K_pad/2]")
    _need(scales.dtype in _DT and scales.is_contiguous(), "repack_weight: scales must be contiguous bf16/fp16/fp32")
    n, k_pad = qweight.shape[0], qweight.shape[1] * 2
    w16 = torch.empty((n, k_pad), dtype=torch.float16, device=qweight.device)
    _lib.call("svdq_repack_weight", _p(qweight), _p(scales), _DT[scales.dtype], n, k_pad, w_group, _p(w16),
              _stream(qweight.device))
    return w16


@repack_weight.register_fake
def _(qweight, scales, w_group):
    return qweight.new_empty((qweight.shape[0], qweight.shape[1] * 2), dtype=torch.float16)


@_op("build_up_hl")
def build_up_hl(l1: Tensor, lora_up: Optional[Tensor], r2: int) -> Tensor:
    """``[up | up | 0]`` with ``up = [l1 | lora_up]`` (bf16) for the fused low-rank MMA."""
    _need_cuda("build_up_hl", l1, lora_up)
    n, rank = l1.shape
    lrank = 0 if lora_up is None else lora_up.shape[1]
    out = torch.empty((n, r2), dtype=torch.bfloat16, device=l1.device)
    _lib.call("svdq_build_up_hl", _p(l1), rank, _p(lora_up), lrank, n, _p(out), r2, _stream(l1.device))
    return out


@build_up_hl.register_fake
def _(l1, lora_up, r2):
    return l1.new_empty((l1.shape[0], r2), dtype=torch.bfloat16)


# --------------------------------------------------------------------------- GEMM
_gemm_ws: "collections.OrderedDict[tuple, Tensor]" = collections.OrderedDict()
_gemm_ws_lock = threading.Lock()


def _gemm_workspace(dev: torch.device) -> Optional[Tensor]:
    """Zero-filled split-tail workspace of ``svdq_linear_gemm_ws``, one per (device, stream).

    Launches on one stream run in order, so a stream's launches share its workspace; each
    launch leaves it ready for the next (the sync words are never re-zeroed).  Inside a CUDA
    graph capture no workspace is used at all (the launch runs unsplit): a captured graph would
    keep the workspace's address after this cache had evicted and freed it."""
    if torch.cuda.is_current_stream_capturing():
        return None
    key = (dev.index, _raw_stream(dev))
    with _gemm_ws_lock:
        ws = _gemm_ws.get(key)
        if ws is not None:
            _gemm_ws.move_to_end(key)
            return ws
        n = int(_lib.lib().svdq_linear_gemm_workspace_bytes())
        ws = torch.zeros((n,), dtype=torch.uint8, device=dev)
        _gemm_ws[key] = ws
        # An evicted workspace returns to the caching allocator, which reuses it only after the
        # work already queued on its stream.
        while len(_gemm_ws) > _GEMM_WS_KEEP:
            _gemm_ws.popitem(last=False)
    return ws


@_op("linear_gemm")
def linear_gemm(a16: Tensor, w16: Tensor, mid_hl: Optional[Tensor], up_hl: Optional[Tensor],
                bias: Optional[Tensor], out_fp32: bool) -> Tensor:
    """``a16 @ w16^T + mid_hl @ up_hl^T + bias`` on tcgen05 CTA pairs (fp32 accumulation)."""
    _need_cuda("linear_gemm", a16, w16, mid_hl, up_hl, bias)
    _need(a16.dtype == torch.float16 and w16.dtype == torch.float16, "linear_gemm: a16/w16 must be fp16")
    m, k_pad = a16.shape
    n = w16.shape[0]
    _need(w16.shape[1] == k_pad, "linear_gemm: activation / weight K mismatch")
    r2 = 0 if mid_hl is None or mid_hl.numel() == 0 else mid_hl.shape[1]
    _need(r2 == 0 or (up_hl is not None and tuple(up_hl.shape) == (n, r2)), "linear_gemm: up_hl shape mismatch")
    out = torch.empty((m, n), dtype=torch.float32 if out_fp32 else torch.bfloat16, device=a16.device)
    if m == 0:
        return out
    ws = _gemm_workspace(a16.device)
    _lib.call("svdq_linear_gemm_ws", _p(a16), _p(w16), _p(mid_hl) if r2 else None, _p(up_hl) if r2 else None, r2,
              _p(bias), _p(out), _lib.SVDQ_FP32 if out_fp32 else _lib.SVDQ_BF16, out.stride(0), m, n, k_pad,
              _p(ws), 0 if ws is None else ws.numel(), _stream(a16.device))
    return out


@linear_gemm.register_fake
def _(a16, w16, mid_hl, up_hl, bias, out_fp32):
    return a16.new_empty((a16.shape[0], w16.shape[0]), dtype=torch.float32 if out_fp32 else torch.bfloat16)


@_op("linear_gemm_small")
def linear_gemm_small(a16: Tensor, w16: Tensor, mid_hl: Optional[Tensor], up_hl: Optional[Tensor],
                      bias: Optional[Tensor], out_fp32: bool) -> Tensor:
    """``linear_gemm`` for small batches (``svdq_linear_gemm_small``: weight rows as the MMA's M,
    tokens as its N, bound by the bytes of w16)."""
    _need_cuda("linear_gemm_small", a16, w16, mid_hl, up_hl, bias)
    _need(a16.dtype == torch.float16 and w16.dtype == torch.float16, "linear_gemm_small: a16/w16 must be fp16")
    m, k_pad = a16.shape
    n = w16.shape[0]
    _need(w16.shape[1] == k_pad, "linear_gemm_small: activation / weight K mismatch")
    r2 = 0 if mid_hl is None or mid_hl.numel() == 0 else mid_hl.shape[1]
    _need(r2 == 0 or (up_hl is not None and tuple(up_hl.shape) == (n, r2)), "linear_gemm_small: up_hl shape mismatch")
    out = torch.empty((m, n), dtype=torch.float32 if out_fp32 else torch.bfloat16, device=a16.device)
    if m == 0:
        return out
    _lib.call("svdq_linear_gemm_small", _p(a16), _p(w16), _p(mid_hl) if r2 else None, _p(up_hl) if r2 else None, r2,
              _p(bias), _p(out), _lib.SVDQ_FP32 if out_fp32 else _lib.SVDQ_BF16, out.stride(0), m, n, k_pad,
              _stream(a16.device))
    return out


@linear_gemm_small.register_fake
def _(a16, w16, mid_hl, up_hl, bias, out_fp32):
    return a16.new_empty((a16.shape[0], w16.shape[0]), dtype=torch.float32 if out_fp32 else torch.bfloat16)


EPILOGUES = {"add": _lib.SVDQ_EPI_ADD, "sigmoid_mul": _lib.SVDQ_EPI_SIGMOID_MUL, "silu_mul": _lib.SVDQ_EPI_SILU_MUL}


@_op("linear_gemm_epi")
def linear_gemm_epi(a16: Tensor, w16: Tensor, mid_hl: Optional[Tensor], up_hl: Optional[Tensor],
                    bias: Optional[Tensor], out_fp32: bool, epilogue: int, aux: Tensor) -> Tensor:
    """``linear_gemm`` whose epilogue combines its output y with ``aux`` (z, [M, N] in the output
    dtype): ``z + y``, ``z * sigmoid(y)`` or ``silu(z) * y`` (``EPILOGUES``)."""
    _need_cuda("linear_gemm_epi", a16, w16, mid_hl, up_hl, bias, aux)
    _need(a16.dtype == torch.float16 and w16.dtype == torch.float16, "linear_gemm_epi: a16/w16 must be fp16")
    m, k_pad = a16.shape
    n = w16.shape[0]
    _need(w16.shape[1] == k_pad, "linear_gemm_epi: activation / weight K mismatch")
    r2 = 0 if mid_hl is None or mid_hl.numel() == 0 else mid_hl.shape[1]
    _need(r2 == 0 or (up_hl is not None and tuple(up_hl.shape) == (n, r2)), "linear_gemm_epi: up_hl shape mismatch")
    out_dtype = torch.float32 if out_fp32 else torch.bfloat16
    _need(aux.dtype == out_dtype and aux.dim() == 2 and tuple(aux.shape) == (m, n) and aux.stride(1) == 1,
          "linear_gemm_epi: aux must be [M, N] in the output dtype with unit column stride")
    out = torch.empty((m, n), dtype=out_dtype, device=a16.device)
    if m == 0:
        return out
    ws = _gemm_workspace(a16.device)
    _lib.call("svdq_linear_gemm_epi", _p(a16), _p(w16), _p(mid_hl) if r2 else None, _p(up_hl) if r2 else None, r2,
              _p(bias), int(epilogue), _p(aux), aux.stride(0), _p(out),
              _lib.SVDQ_FP32 if out_fp32 else _lib.SVDQ_BF16, out.stride(0), m, n, k_pad,
              _p(ws), 0 if ws is None else ws.numel(), _stream(a16.device))
    return out


@linear_gemm_epi.register_fake
def _(a16, w16, mid_hl, up_hl, bias, out_fp32, epilogue, aux):
    return a16.new_empty((a16.shape[0], w16.shape[0]), dtype=torch.float32 if out_fp32 else torch.bfloat16)


@_op("linear_gemm_group")
def linear_gemm_group(a16: list[Tensor], w16: list[Tensor], mid_hl: list[Optional[Tensor]],
                      up_hl: list[Optional[Tensor]], bias: list[Optional[Tensor]], out_fp32: bool) -> list[Tensor]:
    """Up to four ``linear_gemm`` problems sharing M, K_pad and the low-rank width R2 as one
    persistent launch (``svdq_linear_gemm_group``)."""
    n_p = len(a16)
    _need(1 <= n_p <= 4 and len(w16) == n_p and len(mid_hl) == n_p and len(up_hl) == n_p and len(bias) == n_p,
          "linear_gemm_group: 1 to 4 problems with one entry per list")
    _need_cuda("linear_gemm_group", *a16, *w16, *mid_hl, *up_hl, *bias)
    m, k_pad = a16[0].shape
    r2s = {0 if t is None or t.numel() == 0 else t.shape[1] for t in mid_hl}
    _need(len(r2s) == 1, "linear_gemm_group: every problem needs the same low-rank width R2")
    r2 = r2s.pop()
    dev = a16[0].device
    probs = (_lib.GemmProblem * n_p)()
    outs = []
    for i in range(n_p):
        a, w = a16[i], w16[i]
        _need(a.dtype == torch.float16 and w.dtype == torch.float16, "linear_gemm_group: a16/w16 must be fp16")
        _need(tuple(a.shape) == (m, k_pad) and w.shape[1] == k_pad, "linear_gemm_group: M / K_pad mismatch")
        n = w.shape[0]
        _need(r2 == 0 or (up_hl[i] is not None and tuple(up_hl[i].shape) == (n, r2)),
              "linear_gemm_group: up_hl shape mismatch")
        out = torch.empty((m, n), dtype=torch.float32 if out_fp32 else torch.bfloat16, device=dev)
        outs.append(out)
        probs[i] = _lib.GemmProblem(a.data_ptr(), w.data_ptr(), mid_hl[i].data_ptr() if r2 else None,
                                    up_hl[i].data_ptr() if r2 else None,
                                    None if bias[i] is None else bias[i].data_ptr(), 0, None, 0,
                                    out.data_ptr(), out.stride(0), n)
    if m == 0:
        return outs
    ws = _gemm_workspace(dev)
    _lib.call("svdq_linear_gemm_group", probs, n_p, r2, _lib.SVDQ_FP32 if out_fp32 else _lib.SVDQ_BF16, m, k_pad,
              _p(ws), 0 if ws is None else ws.numel(), _stream(dev))
    return outs


@linear_gemm_group.register_fake
def _(a16, w16, mid_hl, up_hl, bias, out_fp32):
    dt = torch.float32 if out_fp32 else torch.bfloat16
    return [a.new_empty((a.shape[0], w.shape[0]), dtype=dt) for a, w in zip(a16, w16)]


def apply_epilogue(y: Tensor, epilogue: Optional[tuple[str, Tensor]]) -> Tensor:
    """The unfused form of an epilogue operation, as torch ops on the linear's output ``y``: the
    sequence the fused GEMM epilogue reproduces."""
    if epilogue is None:
        return y
    op, z = epilogue
    z = z.reshape(y.shape)
    if op == "add":
        return z + y
    if op == "sigmoid_mul":
        return z * torch.sigmoid(y)
    if op == "silu_mul":
        return torch.nn.functional.silu(z) * y
    raise ValueError(f"unknown epilogue operation {op!r}; expected one of {sorted(EPILOGUES)}")


# --------------------------------------------------------------------------- packed-weight GEMM
@_op("prepare_packed")
def prepare_packed(qweight: Tensor, scales: Tensor, w_group: int) -> tuple[Tensor, Tensor, Tensor]:
    """Checkpoint INT4 weight -> the packed-weight GEMM's operands: ``codes [N, K_pad/2]`` u8 in the
    kernel's nibble order, ``scales16`` fp16 in the kernel's tile order (``packed_scales_numel``
    elements: per 128-row tile and 256-k code group, [128 rows][256 / w_group]), and a one-element
    int32 flag that is
    1 when some scale (or its sixteenth) is not an fp16 value (the GEMM's weights then differ from
    ``repack_weight``'s by one more rounding of the scale)."""
    _need_cuda("prepare_packed", qweight, scales)
    _need(qweight.dtype == torch.uint8 and qweight.dim() == 2 and qweight.is_contiguous(),
          "prepare_packed: qweight must be contiguous uint8 [N, K_pad/2]")
    _need(scales.dtype in _DT and scales.is_contiguous(), "prepare_packed: scales must be contiguous bf16/fp16/fp32")
    n, k_pad = qweight.shape[0], qweight.shape[1] * 2
    codes = torch.empty_like(qweight)
    scales16 = torch.empty((packed_scales_numel(n, k_pad, w_group),), dtype=torch.float16, device=qweight.device)
    flag = torch.zeros((1,), dtype=torch.int32, device=qweight.device)
    _lib.call("svdq_prepare_packed", _p(qweight), _p(scales), _DT[scales.dtype], n, k_pad, w_group, _p(codes),
              _p(scales16), _p(flag), _stream(qweight.device))
    return codes, scales16, flag


@prepare_packed.register_fake
def _(qweight, scales, w_group):
    n, k_pad = qweight.shape[0], qweight.shape[1] * 2
    return (torch.empty_like(qweight), qweight.new_empty((packed_scales_numel(n, k_pad, w_group),),
                                                         dtype=torch.float16),
            qweight.new_empty((1,), dtype=torch.int32))


PACKED_GROUP_SIZES = (32, 64, 128, 256)


def packed_scales_numel(n: int, k_pad: int, w_group: int) -> int:
    """Elements of the packed GEMM's tile-ordered fp16 scales: per 128-row tile and 256-k code group,
    [128 rows][256 / w_group] (padded with zeros past N and K_pad)."""
    return -(-n // 128) * -(-k_pad // 256) * 128 * (256 // w_group)


@_op("packed_gemm")
def packed_gemm(a16: Tensor, codes: Tensor, scales16: Tensor, w_group: int, mid_hl: Optional[Tensor],
                up_hl: Optional[Tensor], bias: Optional[Tensor], out_fp32: bool) -> Tensor:
    """``a16 @ (q * s)^T + mid_hl @ up_hl^T + bias`` with the weight read as packed codes and converted
    to fp16 in shared memory (tcgen05, fp32 accumulation)."""
    _need_cuda("packed_gemm", a16, codes, scales16, mid_hl, up_hl, bias)
    _need(a16.dtype == torch.float16 and a16.is_contiguous(), "packed_gemm: a16 must be contiguous fp16")
    _need(codes.dtype == torch.uint8 and scales16.dtype == torch.float16, "packed_gemm: codes u8, scales16 fp16")
    m, k_pad = a16.shape
    n = codes.shape[0]
    _need(codes.shape[1] * 2 == k_pad, "packed_gemm: activation / weight K mismatch")
    r2 = 0 if mid_hl is None or mid_hl.numel() == 0 else mid_hl.shape[1]
    _need(r2 == 0 or (up_hl is not None and tuple(up_hl.shape) == (n, r2)), "packed_gemm: up_hl shape mismatch")
    out = torch.empty((m, n), dtype=torch.float32 if out_fp32 else torch.bfloat16, device=a16.device)
    if m == 0:
        return out
    _lib.call("svdq_packed_gemm", _p(a16), _p(codes), _p(scales16), w_group, _p(mid_hl) if r2 else None,
              _p(up_hl) if r2 else None, r2, _p(bias), _p(out), _lib.SVDQ_FP32 if out_fp32 else _lib.SVDQ_BF16,
              out.stride(0), m, n, k_pad, _stream(a16.device))
    return out


@packed_gemm.register_fake
def _(a16, codes, scales16, w_group, mid_hl, up_hl, bias, out_fp32):
    return a16.new_empty((a16.shape[0], codes.shape[0]), dtype=torch.float32 if out_fp32 else torch.bfloat16)


@_op("w4a4_gemm")
def w4a4_gemm(codes8: Tensor, ascales: Tensor, a_group: int, codes: Tensor, scales16: Tensor, w_group: int,
              mid_hl: Optional[Tensor], up_hl: Optional[Tensor], bias: Optional[Tensor], out_fp32: bool) -> Tensor:
    """W4A4 GEMM with kind::i8 tensor-core MMAs on int8 codes (``act_quant_i8``) and the packed weight
    (``prepare_packed``): per-group int32 partials rescaled by weight and activation scales, plus
    ``mid_hl @ up_hl^T + bias``.  Meant for batches up to 64 tokens."""
    _need_cuda("w4a4_gemm", codes8, ascales, codes, scales16, mid_hl, up_hl, bias)
    _need(codes8.dtype == torch.int8 and codes8.is_contiguous(), "w4a4_gemm: codes8 must be contiguous int8")
    _need(ascales.dtype == torch.float32 and ascales.is_contiguous(), "w4a4_gemm: ascales must be contiguous fp32")
    m, k_pad = codes8.shape
    n = codes.shape[0]
    _need(codes.shape[1] * 2 == k_pad, "w4a4_gemm: activation / weight K mismatch")
    r2 = 0 if mid_hl is None or mid_hl.numel() == 0 else mid_hl.shape[1]
    _need(r2 == 0 or (up_hl is not None and tuple(up_hl.shape) == (n, r2)), "w4a4_gemm: up_hl shape mismatch")
    out = torch.empty((m, n), dtype=torch.float32 if out_fp32 else torch.bfloat16, device=codes8.device)
    if m == 0:
        return out
    _lib.call("svdq_w4a4_gemm", _p(codes8), _p(ascales), ascales.shape[1], a_group, _p(codes), _p(scales16), w_group,
              _p(mid_hl) if r2 else None, _p(up_hl) if r2 else None, r2, _p(bias), _p(out),
              _lib.SVDQ_FP32 if out_fp32 else _lib.SVDQ_BF16, out.stride(0), m, n, k_pad, _stream(codes8.device))
    return out


@w4a4_gemm.register_fake
def _(codes8, ascales, a_group, codes, scales16, w_group, mid_hl, up_hl, bias, out_fp32):
    return codes8.new_empty((codes8.shape[0], codes.shape[0]), dtype=torch.float32 if out_fp32 else torch.bfloat16)


def w4a4_narrow_ok(m: int, n: int, k_pad: int, a_group: int, w_group: int) -> bool:
    """Whether ``w4a4_gemm_narrow`` takes this shape (``svdq_w4a4_gemm_narrow``'s requirements)."""
    return 0 < m <= 16 and n % 128 == 0 and k_pad % 512 == 0 and a_group == 64 and w_group == 64


@_op("w4a4_gemm_narrow")
def w4a4_gemm_narrow(codes8: Tensor, ascales: Tensor, a_group: int, codes: Tensor, scales16: Tensor, w_group: int,
                     mid_hl: Optional[Tensor], up_hl: Optional[Tensor], bias: Optional[Tensor],
                     out_fp32: bool) -> Tensor:
    """``w4a4_gemm`` for up to 16 tokens on mma.sync int8 fragments in registers, K split over a CTA
    pair; same operands and result, the fp32 sums in another order."""
    _need_cuda("w4a4_gemm_narrow", codes8, ascales, codes, scales16, mid_hl, up_hl, bias)
    _need(codes8.dtype == torch.int8 and codes8.is_contiguous(), "w4a4_gemm_narrow: codes8 must be contiguous int8")
    _need(ascales.dtype == torch.float32 and ascales.is_contiguous(), "w4a4_gemm_narrow: ascales must be contiguous fp32")
    m, k_pad = codes8.shape
    n = codes.shape[0]
    _need(codes.shape[1] * 2 == k_pad, "w4a4_gemm_narrow: activation / weight K mismatch")
    r2 = 0 if mid_hl is None or mid_hl.numel() == 0 else mid_hl.shape[1]
    _need(r2 == 0 or (up_hl is not None and tuple(up_hl.shape) == (n, r2)), "w4a4_gemm_narrow: up_hl shape mismatch")
    out = torch.empty((m, n), dtype=torch.float32 if out_fp32 else torch.bfloat16, device=codes8.device)
    if m == 0:
        return out
    _lib.call("svdq_w4a4_gemm_narrow", _p(codes8), _p(ascales), ascales.shape[1], a_group, _p(codes), _p(scales16),
              w_group, _p(mid_hl) if r2 else None, _p(up_hl) if r2 else None, r2, _p(bias), _p(out),
              _lib.SVDQ_FP32 if out_fp32 else _lib.SVDQ_BF16, out.stride(0), m, n, k_pad, _stream(codes8.device))
    return out


@w4a4_gemm_narrow.register_fake
def _(codes8, ascales, a_group, codes, scales16, w_group, mid_hl, up_hl, bias, out_fp32):
    return codes8.new_empty((codes8.shape[0], codes.shape[0]), dtype=torch.float32 if out_fp32 else torch.bfloat16)


# The plain implementations of the ops above, same names and arguments.
eager = types.SimpleNamespace(**_EAGER)
