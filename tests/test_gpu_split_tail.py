"""Split-tail GEMM (svdq_linear_gemm_ws) through the C ABI against an fp64 PyTorch reference
of the same operands, against the unsplit kernel, and against itself (determinism and
reuse of one workspace across launches of different grids)."""
from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _lib_ready():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from krea2_svdquant_b200 import _lib, build
    build.build()
    _lib.lib()
    yield
    assert _lib.device_error() == 0


def _P(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _schedule(m, n, k_pad, r2, ws):
    from krea2_svdquant_b200 import _lib
    out = (ctypes.c_int * 4)()
    assert _lib.lib().svdq_linear_gemm_schedule(m, n, k_pad, r2, 1 if ws else 0, out) == 0
    return tuple(out)


def _operands(m, n, k_pad, r2, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    # fp16 values with few significant bits, like q * scale
    a16 = (torch.randint(-8, 8, (m, k_pad), device="cuda", generator=g).float() * 0.03125).half()
    w16 = (torch.randint(-8, 8, (n, k_pad), device="cuda", generator=g).float() * 0.0078125).half()
    mid = (torch.randn(m, r2, device="cuda", generator=g) * 0.5).bfloat16() if r2 else None
    up = (torch.randn(n, r2, device="cuda", generator=g) * 0.05).bfloat16() if r2 else None
    bias = (torch.randn(n, device="cuda", generator=g) * 0.1).bfloat16()
    return a16, w16, mid, up, bias


def _reference(a16, w16, mid, up, bias):
    y = a16.double() @ w16.double().T
    if mid is not None:
        y += mid.double() @ up.double().T
    return y + bias.double()


def _gemm(a16, w16, mid, up, bias, out_fp32, ws=None):
    from krea2_svdquant_b200 import _lib
    m, k_pad = a16.shape
    n = w16.shape[0]
    r2 = 0 if mid is None else mid.shape[1]
    out = torch.empty(m, n, device="cuda", dtype=torch.float32 if out_fp32 else torch.bfloat16)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    L = _lib.lib()
    dt = _lib.SVDQ_FP32 if out_fp32 else _lib.SVDQ_BF16
    if ws is None:
        st = L.svdq_linear_gemm(_P(a16), _P(w16), _P(mid), _P(up), r2, _P(bias), _P(out), dt, n, m, n, k_pad, stream)
    else:
        st = L.svdq_linear_gemm_ws(_P(a16), _P(w16), _P(mid), _P(up), r2, _P(bias), _P(out), dt, n, m, n, k_pad,
                                   _P(ws), ws.numel(), stream)
    assert st == 0, L.svdq_last_error().decode()
    return out


def _workspace():
    from krea2_svdquant_b200 import _lib
    return torch.zeros(int(_lib.lib().svdq_linear_gemm_workspace_bytes()), dtype=torch.uint8, device="cuda")


SHAPES = [
    # M, N, K_pad, R2, fp32 out   (tiles of 256 x 256; the block shapes have M = 4352)
    (4352, 1536, 6144, 64, True),     # to_k / to_v: one whole wave + a 28-tile split tail
    (4352, 6144, 6144, 64, False),    # to_q / to_gate / to_out.0: five waves + 38 tiles
    (4352, 6144, 16384, 64, False),   # ff.down: long K
    (256, 256, 1024, 64, True),       # a single tile cut into three K ranges (8 + 8 + 1)
    (512, 512, 6144, 128, True),      # four tiles, four ranges each: owners add three partials
    (300, 520, 640, 0, True),         # ragged rows and columns, no low-rank term
]


@pytest.mark.parametrize("m,n,k_pad,r2,out_fp32", SHAPES)
def test_split_tail_matches_reference(m, n, k_pad, r2, out_fp32):
    pairs, dp_tiles, tail_len, tail_total = _schedule(m, n, k_pad, r2, True)
    assert tail_total > 0 and 0 < tail_len < k_pad // 64 + r2 // 64, "shape must exercise the split tail"
    assert _schedule(m, n, k_pad, r2, False)[3] == 0
    ops = _operands(m, n, k_pad, r2, seed=m + n + k_pad)
    ws = _workspace()
    y = _gemm(*ops, out_fp32, ws)
    y_whole = _gemm(*ops, out_fp32)
    ref = _reference(*ops)
    torch.cuda.synchronize()
    if out_fp32:
        # fp32 accumulation in another order: differences at the level of fp32 rounding
        rel = ((y.double() - ref).norm() / ref.norm()).item()
        assert rel < 1e-5, rel
        rel_w = ((y.double() - y_whole.double()).norm() / ref.norm()).item()
        assert rel_w < 1e-5, rel_w
    else:
        # bf16 outputs: within one bf16 rounding of the exact value
        err = (y.double() - ref).abs()
        assert (err <= ref.abs() * 2.0 ** -8 + 1e-5).all()
    # deterministic: the same launch again through the same workspace
    y2 = _gemm(*ops, out_fp32, ws)
    torch.cuda.synchronize()
    assert torch.equal(y, y2)


def test_one_workspace_across_grids_and_launches():
    """Launches of different grid sizes alternate on one workspace; the generation
    counter keeps every launch's flags apart, so each result repeats bit for bit."""
    ws = _workspace()
    cases = [(256, 256, 1024, 64), (4352, 1536, 6144, 64), (300, 520, 640, 0), (512, 512, 6144, 128)]
    first = {}
    inputs = {c: _operands(*c, seed=7) for c in cases}
    for rep in range(3):
        for c in cases:
            y = _gemm(*inputs[c], True, ws)
            if rep == 0:
                first[c] = y
            else:
                assert torch.equal(y, first[c])
    torch.cuda.synchronize()
    # sync words: generation advanced once per split launch, CTA counter back to zero
    sync = ws[:8].view(torch.int32).cpu()
    assert int(sync[1]) == 0
    assert int(sync[0]) == 3 * len(cases)


def test_unsplit_shapes_keep_the_plain_schedule():
    # tails of more than 4/5 of a wave, and tiles with too few K iterations, stay unsplit
    from krea2_svdquant_b200 import _lib
    pairs = _schedule(4352, 16384, 6144, 64, False)[0]
    m_blocks = 17
    assert _schedule(256, 256, 256, 0, True)[3] == 0            # 4 K iterations
    assert _schedule(4352, 16384, 6144, 64, True)[3] == (0 if (m_blocks * 64) % pairs * 20 > pairs * 11 else
                                                         (m_blocks * 64) % pairs * 97)
    assert _schedule(512, 6144, 6144, 64, True)[3] == 0          # 48 tiles: a last wave of 0.65
    assert _lib.lib().svdq_linear_gemm_workspace_bytes() > 0


def test_module_path_uses_split_tail_and_matches_oracle_tolerance():
    """SVDQuantLinear goes through ops.linear_gemm, which passes a per-stream workspace."""
    from krea2_svdquant_b200 import ops
    a16, w16, mid, up, bias = _operands(256, 256, 1024, 64, seed=3)
    y = ops.linear_gemm(a16, w16, mid, up, bias, True)
    ref = _reference(a16, w16, mid, up, bias)
    torch.cuda.synchronize()
    assert ((y.double() - ref).norm() / ref.norm()).item() < 1e-5
    # under graph capture no workspace is used, even one the stream already has: the captured
    # launch runs unsplit
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        y_eager = ops.linear_gemm(a16, w16, mid, up, bias, True)  # creates the stream's workspace
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            yg = ops.linear_gemm(a16, w16, mid, up, bias, True)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(yg, _gemm(a16, w16, mid, up, bias, True))
    assert torch.equal(y_eager, y)
