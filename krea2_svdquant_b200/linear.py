"""``SVDQuantLinear``: drop-in module for src/krea2_svdquant/runtime/linear.py:62-161.

Same constructor, buffers (``smooth_scale, qweight, weight_scales, l1, l2[,
bias]``), attributes, ``add_lora_adapter``, ``state`` property and
``_forward_base`` / ``forward`` split.  The forward runs on the B200 CUDA
library only:

* ``b200`` (W4A4, the default): one activation pass (smoothing, dynamic INT4
  codes per token and group, low-rank + LoRA down-projection) and one fused
  tcgen05 GEMM.  The GEMM's operands are the dequantized codes ``q * scale``
  of activations and weights, both exact in fp16, so the whole K reduction
  accumulates in TMEM; the low-rank/LoRA up-projection, bias and cast are
  fused into the same kernel.
* ``b200_w4a16``: the activation pass only smooths (``fp16(x / s)``), the same
  GEMM runs against the INT4 weight's exact fp16 dequantization.

Errors raise; nothing falls back to another implementation (the reference
swallows kernel errors and reruns its simulation, linear.py:133-154).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import torch
import torch.nn.functional as F
from torch import nn

from . import _lib, ops
from .config import BackendKind, resolve_backend
from .quant import SVDQuantLinearState


class SVDQuantLoRAAdapter(nn.Module):
    """Inference-only LoRA branch (linear.py:11-45): ``(x @ down^T) @ up^T * multiplier``
    with ``multiplier = scale * network_alpha / rank``.  Inside
    :class:`SVDQuantLinear` the branch is fused into the CUDA kernels; this
    module's own ``forward`` exists for API parity."""

    def __init__(self, down_weight: torch.Tensor, up_weight: torch.Tensor, *, scale: float = 1.0,
                 network_alpha: float | None = None) -> None:
        super().__init__()
        if down_weight.ndim != 2 or up_weight.ndim != 2:
            raise ValueError("LoRA down/up weights must be rank-2 tensors")
        rank = int(down_weight.shape[0])
        if rank <= 0:
            raise ValueError("LoRA rank must be positive")
        if int(up_weight.shape[1]) != rank:
            raise ValueError(f"LoRA shape mismatch: down={tuple(down_weight.shape)} up={tuple(up_weight.shape)}")
        self.rank = rank
        self.scale = float(scale)
        self.network_alpha = float(network_alpha) if network_alpha is not None else float(rank)
        self.register_buffer("down_weight", down_weight.contiguous(), persistent=True)
        self.register_buffer("up_weight", up_weight.contiguous(), persistent=True)

    @property
    def multiplier(self) -> float:
        return self.scale * (self.network_alpha / self.rank)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        down = self.down_weight.to(dtype=x.dtype)
        up = self.up_weight.to(dtype=x.dtype)
        return F.linear(F.linear(x, down), up) * self.multiplier


@dataclass
class PreparedOperands:
    """Device-resident operands derived once from the checkpoint buffers."""

    device: torch.device
    key: tuple
    k_in: int        # activation width the kernels read (original in_features rounded up to 8)
    k_pad: int       # padded K of the checkpoint
    n: int
    smooth: torch.Tensor           # [k_in] bf16 (padded with ones)
    l2: torch.Tensor | None        # [r8, k_in] bf16
    l2_f16: torch.Tensor | None    # [r8, k_in] fp16 copy (W4A16 activation pass)
    lora_down: torch.Tensor | None  # [rl8, k_in] bf16, stacked adapters
    lora_col_scale: torch.Tensor | None  # [rl8] fp32 multiplier per stacked row
    up_hl: torch.Tensor | None     # [n, R2] bf16, [l1 | lora_up] hi/lo operand
    up_hl_base: torch.Tensor | None  # same without the LoRA columns (for _forward_base)
    w16: torch.Tensor | None       # [n, k_pad] fp16 = q * weight scale (weight_operand "fp16")
    codes: torch.Tensor | None     # [n, k_pad/2] u8 kernel-order codes (weight_operand "packed")
    scales16: torch.Tensor | None  # fp16 group scales in the packed GEMM's tile order (with codes)
    bias: torch.Tensor | None      # [n] bf16


def _kernels():
    """The op implementations for a forward: the plain functions in eager mode (no dispatcher on
    the host's critical path), the registered custom ops while ``torch.compile`` traces."""
    return ops if torch.compiler.is_compiling() else ops.eager


def _pad_rows(t: torch.Tensor, rows: int) -> torch.Tensor:
    return t if t.shape[0] == rows else F.pad(t, (0, 0, 0, rows - t.shape[0]))


def _pad_cols(t: torch.Tensor, cols: int, value: float = 0.0) -> torch.Tensor:
    return t if t.shape[-1] == cols else F.pad(t, (0, cols - t.shape[-1]), value=value)


class SVDQuantLinear(nn.Module):
    """Runtime SVDQuant linear on the B200 kernels (see module docstring).

    ``check_device_errors`` (class default False): after every forward, synchronize and raise
    :class:`~krea2_svdquant_b200._lib.DeviceWaitError` if a bounded in-kernel wait gave up (for
    example when another stream's long kernels kept a split GEMM's CTA pairs from running
    together for seconds).  Off by default because it synchronizes; production callers that
    leave it off should poll ``_lib.raise_on_device_error`` (``svdq_device_error``) once per step.
    """

    check_device_errors = False
    # "fp16" (default): the load-time fp16 weight q * s (4x the packed bytes) and the fp16-weight
    # GEMM, the faster one at every batch size measured; "packed": only the kernel-order codes and
    # fp16 scales (no fp16 weight is allocated: a quarter of the weight memory) and the
    # packed-weight GEMM, which converts the codes on chip.
    WEIGHT_OPERANDS = ("fp16", "packed")

    def __init__(self, state: SVDQuantLinearState, backend: BackendKind | str = BackendKind.AUTO,
                 *, act_group_size: int = 64, weight_operand: str = "fp16"):
        super().__init__()
        self.backend = resolve_backend(backend)
        if weight_operand not in self.WEIGHT_OPERANDS:
            raise ValueError(f"weight_operand must be one of {self.WEIGHT_OPERANDS}, got {weight_operand!r}")
        self.weight_operand = weight_operand
        self.group_size = int(state.group_size)
        self.original_shape = tuple(int(v) for v in state.original_shape)
        self.qweight_packed = bool(state.qweight_packed)
        self.padded_in_features = state.padded_in_features
        self.act_group_size = int(act_group_size)
        self.output_fp32 = False  # fp32-output mode (parity checks); default output dtype follows x
        self.register_buffer("smooth_scale", state.smooth_scale.contiguous(), persistent=True)
        self.register_buffer("qweight", state.qweight.contiguous(), persistent=True)
        self.register_buffer("weight_scales", state.weight_scales.contiguous(), persistent=True)
        self.register_buffer("l1", state.l1.contiguous(), persistent=True)
        self.register_buffer("l2", state.l2.contiguous(), persistent=True)
        if state.bias is None:
            self.bias = None
        else:
            self.register_buffer("bias", state.bias.contiguous(), persistent=True)
        self.lora_adapters = nn.ModuleList()
        self._prepared: PreparedOperands | None = None

    # ------------------------------------------------------------------ reference API
    def add_lora_adapter(self, down_weight: torch.Tensor, up_weight: torch.Tensor, *, scale: float = 1.0,
                         network_alpha: float | None = None) -> None:
        """Attach an inference LoRA adapter (linear.py:88-111)."""
        expected_out, expected_in = self.original_shape
        if tuple(down_weight.shape[1:]) != (expected_in,):
            raise ValueError(f"LoRA down input mismatch for SVDQuantLinear: expected {expected_in}, "
                             f"got {tuple(down_weight.shape)}")
        if int(up_weight.shape[0]) != expected_out:
            raise ValueError(f"LoRA up output mismatch for SVDQuantLinear: expected {expected_out}, "
                             f"got {tuple(up_weight.shape)}")
        self.lora_adapters.append(SVDQuantLoRAAdapter(down_weight, up_weight, scale=scale,
                                                      network_alpha=network_alpha))
        self._prepared = None

    @property
    def state(self) -> SVDQuantLinearState:
        return SVDQuantLinearState(smooth_scale=self.smooth_scale, qweight=self.qweight,
                                   weight_scales=self.weight_scales, l1=self.l1, l2=self.l2, bias=self.bias,
                                   group_size=self.group_size, original_shape=self.original_shape,
                                   qweight_packed=self.qweight_packed,
                                   padded_in_features=self.padded_in_features)

    @property
    def k_pad(self) -> int:
        if self.padded_in_features:
            return int(self.padded_in_features)
        return int(self.qweight.shape[-1]) * (2 if self.qweight_packed else 1)

    # ------------------------------------------------------------------ operand preparation
    def _operand_key(self, device: torch.device) -> tuple:
        bufs = [self.smooth_scale, self.qweight, self.weight_scales, self.l1, self.l2, self.bias]
        for a in self.lora_adapters:
            bufs += [a.down_weight, a.up_weight]
        # the version counter changes on every in-place write (load_state_dict copies into the
        # existing buffers), so updated weights are re-derived rather than served stale
        return (device, self.weight_operand) + tuple(
            (None if b is None else (b.data_ptr(), b.device, b._version)) for b in bufs) + tuple(
            a.multiplier for a in self.lora_adapters)

    def prepare(self, device: torch.device | str | None = None) -> PreparedOperands:
        """Derive (once per device and buffer set) the kernel operands: the fp16
        weight operand ``w16 = q * weight_scale`` and/or the packed-weight GEMM's
        kernel-order codes and fp16 scales (per ``weight_operand``), the ``[l1|lora_up]`` hi/lo
        up-projection operand, padded smoothing / down-projection weights and
        the stacked LoRA down weights with their per-row multipliers."""
        device = torch.device(device) if device is not None else self.qweight.device
        if device.type != "cuda":
            raise ValueError("SVDQuantLinear.prepare needs a CUDA device (no CPU path in this runtime)")
        key = self._operand_key(device)
        if self._prepared is not None and self._prepared.key == key:
            return self._prepared
        if not self.qweight_packed:
            raise ValueError("SVDQuantLinear on b200 expects a packed uint8 qweight (checkpoint format)")
        n, k_orig = self.original_shape
        k_pad = self.k_pad
        k_in = ops.round_up(k_orig, 8)
        if k_in > k_pad:
            raise ValueError(f"padded K {k_pad} is smaller than in_features rounded to 8 ({k_in})")
        if k_pad % 64:
            raise ValueError(f"padded K {k_pad} must be a multiple of 64")
        if self.group_size % 16 or k_pad % self.group_size:
            raise ValueError(f"weight group size {self.group_size} must be a multiple of 16 dividing K_pad")
        bf = torch.bfloat16
        with torch.no_grad():
            smooth = _pad_cols(self.smooth_scale.to(device=device, dtype=bf), k_in, 1.0).contiguous()
            rank = int(self.l1.shape[1])
            r8 = ops.round_up(rank, 8)
            l2 = None
            l1p = None
            if rank > 0:
                l2 = _pad_rows(_pad_cols(self.l2.to(device=device, dtype=bf), k_in), r8).contiguous()
                l1p = _pad_cols(self.l1.to(device=device, dtype=bf), r8).contiguous()
            downs, ups, cscale = [], [], []
            for a in self.lora_adapters:
                rl8 = ops.round_up(a.rank, 8)
                downs.append(_pad_rows(_pad_cols(a.down_weight.to(device=device, dtype=bf), k_in), rl8))
                ups.append(_pad_cols(a.up_weight.to(device=device, dtype=bf), rl8))
                cscale.append(torch.full((rl8,), a.multiplier, dtype=torch.float32, device=device))
            lora_down = torch.cat(downs).contiguous() if downs else None
            lora_up = torch.cat(ups, dim=1).contiguous() if ups else None
            col_scale = torch.cat(cscale).contiguous() if cscale else None
            r_tot = (r8 if rank > 0 else 0) + (0 if lora_down is None else lora_down.shape[0])
            r2 = ops.lowrank_width(r_tot)
            l1_in = l1p if l1p is not None else torch.zeros((n, 0), dtype=bf, device=device)
            up_hl = ops.build_up_hl(l1_in, lora_up, r2) if r2 else None
            up_hl_base = up_hl
            if lora_up is not None:
                r2b = ops.lowrank_width(r8 if rank > 0 else 0)
                up_hl_base = ops.build_up_hl(l1_in, None, r2b) if r2b else None
            qw = self.qweight.to(device=device).contiguous()
            ws = self.weight_scales.to(device=device).contiguous()
            w16 = codes = scales16 = None
            if self.weight_operand == "fp16":
                w16 = ops.repack_weight(qw, ws, self.group_size)
            else:
                if self.group_size not in ops.PACKED_GROUP_SIZES:
                    raise ValueError(f"the packed-weight GEMM takes weight group sizes {ops.PACKED_GROUP_SIZES}, "
                                     f"got {self.group_size} (use weight_operand='fp16')")
                codes, scales16, _ = ops.prepare_packed(qw, ws, self.group_size)
            bias = None if self.bias is None else self.bias.to(device=device, dtype=bf).contiguous()
        self._prepared = PreparedOperands(device=device, key=key, k_in=k_in, k_pad=k_pad, n=n, smooth=smooth,
                                          l2=l2, l2_f16=None if l2 is None else l2.to(torch.float16),
                                          lora_down=lora_down, lora_col_scale=col_scale, up_hl=up_hl,
                                          up_hl_base=up_hl_base,
                                          w16=w16, codes=codes, scales16=scales16, bias=bias)
        return self._prepared

    # ------------------------------------------------------------------ forward
    def _prologue(self, x: torch.Tensor) -> tuple[PreparedOperands, torch.Size, torch.Tensor, bool]:
        """Checks x and returns (prepared operands, leading shape, x as [M, K_in] bf16 rows the
        activation pass can read, whether the output is fp32)."""
        if not x.is_cuda:
            raise ValueError("SVDQuantLinear (b200) needs CUDA activations; this runtime has no CPU path")
        if x.dtype not in (torch.bfloat16, torch.float32):
            raise TypeError(f"SVDQuantLinear (b200) takes bf16 or fp32 activations, got {x.dtype}")
        k_orig = self.original_shape[1]
        if x.shape[-1] != k_orig:
            raise ValueError(f"expected [..., {k_orig}] activations, got {tuple(x.shape)}")
        p = self.prepare(x.device)
        x2 = x.reshape(-1, k_orig)
        if x2.dtype != torch.bfloat16:
            x2 = x2.to(torch.bfloat16)
        if p.k_in != k_orig or x2.stride(1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
            x2 = _pad_cols(x2, p.k_in).contiguous()
        return p, x.shape[:-1], x2, self.output_fp32 or x.dtype == torch.float32

    def _a16_operands(self, p: PreparedOperands, x2: torch.Tensor, include_lora: bool):
        """The activation pass for the fp16-operand GEMMs: (a16, (mid_hl, up_hl) or (None, None))."""
        lora_down = p.lora_down if include_lora else None
        col_scale = p.lora_col_scale if include_lora else None
        up_hl = p.up_hl if include_lora else p.up_hl_base
        k = _kernels()
        if self.backend is BackendKind.B200_W4A16:
            a16, mid = k.w4a16_prep(x2, p.smooth, p.l2_f16, lora_down, col_scale, p.k_pad)
        else:
            a16, mid, _, _ = k.act_quant(x2, p.smooth, p.l2, lora_down, col_scale, p.k_pad,
                                         self.act_group_size, True, False)
        return a16, ((mid, up_hl) if mid.numel() else (None, None))

    def _run(self, x: torch.Tensor, include_lora: bool,
             epilogue: tuple[str, torch.Tensor] | None = None) -> torch.Tensor:
        p, lead, x2, out_fp32 = self._prologue(x)
        n = self.original_shape[0]
        k = _kernels()
        if self.backend is not BackendKind.B200_W4A16 and p.w16 is None and self._int8_path(x2.shape[0], p):
            # small batch, packed weight: int8 codes and a GEMM with per-group rescale (up to 32
            # tokens on register-resident mma.sync fragments, else tcgen05 kind::i8)
            codes8, ascales, mid = k.act_quant_i8(x2, p.smooth, p.l2, p.lora_down if include_lora else None,
                                                    p.lora_col_scale if include_lora else None, p.k_pad,
                                                    self.act_group_size)
            up_hl = p.up_hl if include_lora else p.up_hl_base
            lowrank = (mid, up_hl) if mid.numel() else (None, None)
            narrow = ops.w4a4_narrow_ok(x2.shape[0], p.codes.shape[0], p.k_pad, self.act_group_size, self.group_size)
            gemm = k.w4a4_gemm_narrow if narrow else k.w4a4_gemm
            y = gemm(codes8, ascales, self.act_group_size, p.codes, p.scales16, self.group_size, *lowrank, p.bias,
                     out_fp32)
            if self.check_device_errors:
                _lib.raise_on_device_error(f"SVDQuantLinear {tuple(self.original_shape)}")
            return ops.apply_epilogue(y.reshape(*lead, n), epilogue)
        a16, lowrank = self._a16_operands(p, x2, include_lora)
        z = self._fusable_operand(epilogue, x2.shape[0], out_fp32) if p.w16 is not None else None
        if z is not None:
            # the combining op runs in the GEMM's epilogue: y never makes a round trip through HBM
            y = k.linear_gemm_epi(a16, p.w16, *lowrank, p.bias, out_fp32, ops.EPILOGUES[epilogue[0]], z)
            epilogue = None
        elif p.w16 is None:
            y = k.packed_gemm(a16, p.codes, p.scales16, self.group_size, *lowrank, p.bias, out_fp32)
        elif self._small_gemm(x2.shape[0]):
            y = k.linear_gemm_small(a16, p.w16, *lowrank, p.bias, out_fp32)
        else:
            y = k.linear_gemm(a16, p.w16, *lowrank, p.bias, out_fp32)
        if self.check_device_errors:
            _lib.raise_on_device_error(f"SVDQuantLinear {tuple(self.original_shape)}")
        return ops.apply_epilogue(y.reshape(*lead, n), epilogue)

    def _fusable_operand(self, epilogue, m: int, out_fp32: bool) -> torch.Tensor | None:
        """The epilogue operand as the fused GEMM epilogue takes it ([M, N] rows, output dtype,
        16-byte aligned rows), or None when the operation has to run unfused."""
        if epilogue is None or self._small_gemm(m):
            return None  # small batches take the small GEMM, which has no epilogue operations
        op, z = epilogue
        n = self.original_shape[0]
        if op not in ops.EPILOGUES or not z.is_cuda or z.numel() != m * n:
            return None
        if z.dtype != (torch.float32 if out_fp32 else torch.bfloat16):
            return None
        z2 = z.reshape(m, n)
        if z2.stride(1) != 1 or z2.stride(0) % 8 or z2.data_ptr() % 16:
            return None
        return z2

    # Small batches take the small-batch fp16-weight GEMM (weight rows as the MMA's M, tokens as its
    # N) instead of the CTA-pair GEMM's 256x256 tiles, where it measured faster on B200 (K6144, L2
    # flushed): always up to 64 tokens (N16384: 45 against 47-57 us; N6144: 29-31 against 35-39;
    # N1536: 16 against 31), up to 128 tokens for N <= 8192 and up to 384 for N <= 2048 (N1536 at
    # 384 tokens: 27 against 35 us).
    SMALL_GEMM_MAX_TOKENS = 384

    def _small_gemm(self, m: int) -> bool:
        n = self.original_shape[0]
        return m <= 64 or (m <= 128 and n <= 8192) or (m <= self.SMALL_GEMM_MAX_TOKENS and n <= 2048)

    # Batches up to this many tokens take the int8-code GEMM when the weight is packed (W4A4).
    # Measured on B200 at K6144 N16384 (GEMM only, L2 flushed): int8 codes 33.8 / 34.6 / 41.4 us
    # at 1 / 16 / 32 tokens against 39.2 / 40.0 / 41.0 us for the packed fp16-operand GEMM; at 48
    # and 64 tokens the fp16-operand GEMM is faster (49.3 against 55.5 us).
    INT8_PATH_MAX_TOKENS = 32

    def _int8_path(self, m: int, p: PreparedOperands) -> bool:
        return (0 < m <= self.INT8_PATH_MAX_TOKENS and p.k_pad % 128 == 0 and self.group_size in (64, 128, 256)
                and self.act_group_size in (64, 128) and p.k_pad % self.act_group_size == 0)

    def _forward_base(self, x: torch.Tensor) -> torch.Tensor:
        """SVDQuant base term (residual + low-rank + bias), without LoRA branches."""
        return self._run(x, include_lora=False)

    def forward(self, x: torch.Tensor, epilogue: tuple[str, torch.Tensor] | None = None) -> torch.Tensor:
        """``y = SVDQuant(x)`` (runtime/linear.py:148-161).  ``epilogue=(op, z)`` also combines y with
        a tensor z of y's shape: ``"add"`` gives ``z + y``, ``"sigmoid_mul"`` ``z * sigmoid(y)``,
        ``"silu_mul"`` ``silu(z) * y`` (the glue after a block's linears).  On the fp16-weight
        GEMM the operation runs in its epilogue; its result equals the unfused torch ops'."""
        if "_forward_base" in self.__dict__:
            # an instance-level override of the base (as the reference's LoRA test does,
            # test_lora_loading.py:60): keep the reference's composition base + adapters
            y = self._forward_base(x)
            for adapter in self.lora_adapters:
                y = y + adapter(x)
            return ops.apply_epilogue(y, epilogue)
        if epilogue is not None and epilogue[0] not in ops.EPILOGUES:
            raise ValueError(f"unknown epilogue operation {epilogue[0]!r}; expected one of {sorted(ops.EPILOGUES)}")
        return self._run(x, include_lora=True, epilogue=epilogue)

    def release_prepared(self) -> None:
        """Drop the derived device operands (they are rebuilt on the next forward)."""
        self._prepared = None

    def extra_repr(self) -> str:
        n, k = self.original_shape
        return (f"in_features={k}, out_features={n}, rank={self.l1.shape[1]}, group_size={self.group_size}, "
                f"backend={self.backend.value}, loras={len(self.lora_adapters)}")


def grouped_forward(layers: Sequence[nn.Module], x: torch.Tensor) -> list[torch.Tensor]:
    """``[layer(x) for layer in layers]`` for layers that read the same activations (a block's q / k
    / v projections, its gated-MLP pair).  When every layer is an ``SVDQuantLinear`` on the
    fp16-weight GEMM with the same padded K and low-rank width, and some layer has fewer than
    ``GROUP_MAX_WAVES`` waves of 256x256 tiles, their GEMMs run as one grouped persistent launch
    (``svdq_linear_gemm_group``, up to four): a layer with few tiles fills the waves of the others
    instead of ending in a ragged wave of its own.  Otherwise, and for layers with forward hooks or
    an overridden ``_forward_base``, the layers run one by one."""
    layers = list(layers)
    if not _groupable(layers, x):
        return [layer(x) for layer in layers]
    k = _kernels()
    outs = []
    for start in range(0, len(layers), 4):
        chunk = layers[start:start + 4]
        a16s, w16s, mids, ups, biases = [], [], [], [], []
        lead, out_fp32 = None, False
        for layer in chunk:
            p, lead, x2, out_fp32 = layer._prologue(x)
            a16, (mid, up) = layer._a16_operands(p, x2, include_lora=True)
            a16s.append(a16)
            w16s.append(p.w16)
            mids.append(mid)
            ups.append(up)
            biases.append(p.bias)
        ys = k.linear_gemm_group(a16s, w16s, mids, ups, biases, out_fp32)
        if any(layer.check_device_errors for layer in chunk):
            _lib.raise_on_device_error(f"grouped SVDQuantLinear {[tuple(l.original_shape) for l in chunk]}")
        outs += [y.reshape(*lead, layer.original_shape[0]) for y, layer in zip(ys, chunk)]
    return outs


# Grouping pays while some layer of the group would end its own launch in a ragged wave that the
# others can fill: measured on B200, q/k/v/gate at 4352 tokens ran 2% faster grouped, q/k/v at
# 34816 tokens 0.8% slower in the 28-block forward (each layer has 11 or more waves of tiles there).
GROUP_MAX_WAVES = 4
_PAIRS: dict[int, int] = {}


def _pairs_per_device(dev: torch.device) -> int:
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    n = _PAIRS.get(idx)
    if n is None:
        n = _PAIRS[idx] = max(1, torch.cuda.get_device_properties(idx).multi_processor_count // 2)
    return n


def _groupable(layers: list[nn.Module], x: torch.Tensor) -> bool:
    if len(layers) < 2 or not x.is_cuda or x.dtype not in (torch.bfloat16, torch.float32):
        return False
    if not all(isinstance(layer, SVDQuantLinear) for layer in layers):
        return False
    m = x.numel() // max(1, x.shape[-1])
    if any(layer._small_gemm(m) for layer in layers):
        return False  # those layers take the small-batch GEMM
    row_blocks = -(-m // 256)
    fewest_tiles = min(row_blocks * -(-layer.original_shape[0] // 256) for layer in layers)
    if fewest_tiles >= GROUP_MAX_WAVES * _pairs_per_device(x.device):
        return False
    keys = set()
    for layer in layers:
        if not isinstance(layer, SVDQuantLinear) or "_forward_base" in layer.__dict__:
            return False
        if layer._forward_hooks or layer._forward_pre_hooks:
            return False
        if x.shape[-1] != layer.original_shape[1]:
            return False
        p = layer.prepare(x.device)
        if p.w16 is None:
            return False
        r2 = 0 if p.up_hl is None else p.up_hl.shape[1]
        keys.add((p.k_pad, r2, layer.output_fp32))
    return len(keys) == 1
