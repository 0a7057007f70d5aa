// Activation pass of the SVDQuant linear (sm_100a).
//
// W4A4 mode, per element of x [M, K_in] bf16:
//   x_hat = bf16(x / smooth)                             (svd.py:122)
//   scale = bf16(max(amax_group(x_hat), bf16(1e-8)) / 7) (pack.py:20)
//   q     = clamp(rint(x_hat / scale), -8, 7)            (pack.py:6-23)
//   packed nibble q + 8, even k in the low nibble        (pack.py:47-56)   [optional output]
//   a16   = fp16(q * scale): the dequantized activation, exact in fp16 (GEMM operand)
//   mid   = [x_hat @ l2^T | (x @ lora_down^T) * col_scale] (svd.py:159, linear.py:45)
// W4A16 mode: a16 = fp16(fp32(x) / fp32(smooth)) (the reference's fp32 run of
// svd.py:122) and mid from that fp16 x_hat against l2 given in fp16.
//
// Work decomposition.  A CTA owns 64 rows (4 warps) or, with 64 or more
// low-rank columns, 128 rows (8 warps) x one K slice (a whole number of
// 64-column stages) x up to 96 low-rank columns; each warp owns 16 rows.  TMA
// brings each stage's x tile (rows x 64) and low-rank rows (8-row boxes) into
// a ring of shared-memory stages with 128-byte swizzle.  A warp
// loads its 16 x 64 x tile straight into mma.sync A-fragment registers with
// ldmatrix and does all per-element work on those registers: the LoRA
// down-projection MMAs on raw x, the division and group quantization, the
// l2 MMAs on x_hat.  a16 leaves through stmatrix into a per-warp swizzled
// staging tile and a TMA store.  Whichever warp releases a stage last refills
// it, so no warp waits on another except through the data itself.
// Low-rank sums of a K slice go to an fp32 workspace; a second launch adds the
// slices in a fixed order (deterministic) and writes the bf16 hi/lo mid.
//
// Exact division without a data-dependent slow path: with y = RN(1/b)
// (__frcp_rn), q0 = RN(a*y), r = fma(-q0, b, a) (exact), q1 = RN(q0 + r*y)
// (Markstein's correction, P. Markstein, IBM J. R&D 34(1), 1990) is the
// correctly rounded quotient RN(a/b).  For bf16 operands this was checked
// exhaustively against IEEE division on sm_100a: the bf16-rounded x_hat agrees
// for every finite x with |x| >= 2^-118 or x == 0 and every normal smooth
// whose quotient stays below 2^126; rint(x_hat / scale) and the /7 of the scale
// agree for all bf16 inputs with a normal scale (the scale is >= 1.4e-9).
// Outside that domain the kernel divides with IEEE division (__fdiv_rn): a warp
// redoes a whole stage that way when one of its elements has 0 < |x| < 2^-118
// or a quotient that is inf, NaN or (bf16) >= 2^126, and a CTA whose slice has
// a zero, subnormal or non-finite smoothing factor does so for every stage.  So
// x_hat (and fp16(x / s) in W4A16 mode) equals IEEE division for every input.
#include <algorithm>
#include <atomic>

#include "svdq_common.cuh"

namespace svdq {
namespace {

// Warps per CTA, each owning 16 rows: 8 (128 rows) with eight or more low-rank tiles, so each
// stage's low-rank boxes serve twice the rows; else 4 (64 rows), which keeps more CTAs per SM.
__host__ __device__ constexpr int cta_warps(int nt) { return nt >= 8 ? 8 : 4; }
__host__ __device__ constexpr int cta_rows(int nt) { return 16 * cta_warps(nt); }
constexpr int kBK = 64;              // columns per stage: one 128-byte swizzle row of bf16
constexpr int kTargetCtasPerSm = 4;
// x / low-rank ring depth and a16 staging tiles per warp (16 rows x 64 columns of fp16 each):
// four stages and two tiles (a warp writes one while the TMA store of the other reads it) without
// a low-rank operand; three stages and one tile with one, so that four 64-row or two 128-row CTAs
// fit an SM and the K split fills one wave.
__host__ __device__ constexpr int ring_stages(int nt) { return nt == 0 ? 4 : 3; }
__host__ __device__ constexpr int out_bufs(int nt) { return nt == 0 ? 2 : 1; }
constexpr uint32_t kOutTileBytes = 16 * 64 * 2;
// Stages per CTA slice, which bounds the reciprocal table: 16 with eight or more low-rank tiles
// (their CTAs fit three per SM either way), else 12 (a 16-stage table would push the CTA past a
// quarter of the SM's shared memory).
__host__ __device__ constexpr int max_slice_stages(int nt) { return nt >= 8 ? 16 : 12; }
// CTAs per SM the launch bound plans registers for.
__host__ __device__ constexpr int min_ctas(int nt) { return nt >= 8 ? 2 : kTargetCtasPerSm; }
constexpr int kMinSliceStages = 2;
// x stage: the CTA's rows x 64 columns of bf16 (8 or 16 KB)
__host__ __device__ constexpr uint32_t x_tile_bytes(int nt) { return (uint32_t)cta_rows(nt) * kBK * 2; }
constexpr uint32_t kLrTileBytes = 8 * kBK * 2;    // 1 KB: 8 low-rank rows
// a16 = q * scale is exact in fp16 while the group scale lies in [2^-17, 65504 / 7]:
// above it a16 overflows (recorded as kErrA16Range in the device error word),
// below it the smallest codes round in fp16's subnormal range (absolute error < 2^-25).
constexpr float kA16ScaleMax = 65504.0f / 7.0f;
constexpr int kErrA16Range = 0x4200;

// ---- fragment-level helpers ----
__device__ __forceinline__ uint32_t swz128(int row, int chunk) {
  return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4));
}
__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void stmatrix_x4(uint32_t addr, uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(r0), "r"(r1),
               "r"(r2), "r"(r3)
               : "memory");
}
template <bool F16>
__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (F16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}
// bf16x2 register (low half = lower column) -> {lo, hi} fp32 pair
__device__ __forceinline__ uint64_t bf2_to_f2(uint32_t v) {
  return f2_pack(__uint_as_float(v << 16), __uint_as_float(v & 0xFFFF0000u));
}
__device__ __forceinline__ uint32_t f2_to_bf2(uint64_t v) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(f2_hi(v)), "f"(f2_lo(v)));
  return d;
}
__device__ __forceinline__ uint32_t f2_to_h2(uint64_t v) {
  uint32_t d;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(f2_hi(v)), "f"(f2_lo(v)));
  return d;
}
// Correctly rounded a / b for a pair, given y = RN(1/b) and nb = -b (Markstein).
__device__ __forceinline__ uint64_t div_f2(uint64_t a, uint64_t y, uint64_t nb) {
  const uint64_t q0 = f2_mul(a, y);
  const uint64_t r = f2_fma(q0, nb, a);
  return f2_fma(r, y, q0);
}
// Where the Markstein quotient above may differ from IEEE division, as bits 15 / 31 of the result
// (other bits are don't-care): x with 0 < |x| < 2^-118 (the residual r loses bits below fp32's
// normal range; tested per element on the bf16x2 input), or a result that is inf / NaN or, in
// bf16, at least 2^126 (the product a * y can overflow; tested on the fp16 output in W4A16 mode
// and on each quantization group's |x_hat| maximum in W4A4 mode, whose max keeps NaNs).  Each
// 16-bit half is tested with one add: h + c sets bit 15 iff h >= 0x8000 - c, and no half carries
// into the next (h <= 0x7FFF).
__device__ __forceinline__ uint32_t tiny_x_lanes(uint32_t xv) {
  const uint32_t t = xv & 0x7FFF7FFFu;
  const uint32_t nonzero = t + 0x7FFF7FFFu;       // bit 15: |x| bits >= 0x0001
  const uint32_t not_tiny = t + 0x7B807B80u;      // bit 15: |x| bits >= 0x0480 (2^-118)
  return nonzero & ~not_tiny;
}
// f16x2: bit 15 / 31 set for inf or NaN; bf16x2: for |v| >= 2^126, inf or NaN
template <bool F16>
__device__ __forceinline__ uint32_t big_lanes(uint32_t v) {
  return (v & 0x7FFF7FFFu) + (F16 ? 0x04000400u : 0x01800180u);
}
__device__ __forceinline__ uint32_t bf162_bits(__nv_bfloat162 v) {
  uint32_t u;
  memcpy(&u, &v, 4);
  return u;
}
// running max of |.| over bf16x2 lanes, NaN if either is NaN (the sign bit of the result is meaningless)
__device__ __forceinline__ uint32_t bf2_maxabs(uint32_t m, uint32_t v) {
  uint32_t d;
  asm("max.NaN.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(m), "r"(v));
  return d;
}

// Non-blocking check of an mbarrier phase.
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Shared-memory counter increment with acquire-release ordering at CTA scope.
__device__ __forceinline__ uint32_t atom_add_acq_rel(uint32_t addr, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], %2;" : "=r"(old) : "r"(addr), "r"(v) : "memory");
  return old;
}

struct AqArgs {
  const __nv_bfloat16* x;  // [M, K_in], row stride ldx (read directly only by the IEEE-division path)
  int64_t ldx;
  int M, K_in, K_pad;
  int rank, lora_rank, r_tot;
  int n_stages;      // K_pad / 64
  int slice_stages;  // stages per CTA along K (the last slice may be shorter)
  int G;             // quantization group (W4A4)
  int write_a16;
  const __nv_bfloat16* smooth;
  uint8_t* packed;        // [M, K_pad/2] or null
  __nv_bfloat16* scales;  // [M, K_pad/G] or null
  int8_t* codes8;         // [M, K_pad] int8 codes q, or null
  float* ascales_t;       // [K_pad/G, lda_s] fp32 scales, group-major, or null
  int64_t lda_s;
  float* partial;         // [ksplit, M, r_tot] or null
  int* err;
};

template <int STAGES, int NT>
__host__ __device__ constexpr uint32_t aq_smem_layout_bytes() {
  return 1024 /*align slack*/ + STAGES * x_tile_bytes(NT) + STAGES * NT * kLrTileBytes +
         cta_warps(NT) * out_bufs(NT) * kOutTileBytes + max_slice_stages(NT) * 32 * 16 /*reciprocal table*/ +
         256 /*barriers, counters*/;
}

// GS: stages per quantization group (1: G=64, 2: G=128).  NT: 8-column
// low-rank tiles per CTA (0: no mid).  PACKED: also write reference-format
// codes and scales.  LORA: some low-rank rows of this launch are LoRA rows
// (multiplied with raw x rather than x_hat).
//
// Each warp writes its 16 x 64 a16 tile in place over its own 16 rows of the
// x stage (the rows it alone reads) and TMA-stores it from there, so a stage
// is released only once that store has read it: stage c is released after
// the store of stage c + 1 is issued (bulk wait_group.read 1), in the same
// single-lane section.
template <int GS, int STAGES, int NT, bool W4A16, bool PACKED, bool LORA>
__global__ void __launch_bounds__(32 * cta_warps(NT), min_ctas(NT))
    act_quant_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_l2,
                     const __grid_constant__ CUtensorMap tm_lora, const __grid_constant__ CUtensorMap tm_a16,
                     const AqArgs a) {
  constexpr int kWarps = cta_warps(NT);
  constexpr int kThreads = 32 * kWarps;
  constexpr int kBM = cta_rows(NT);
  constexpr uint32_t kXTileBytes = x_tile_bytes(NT);
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t xs = base;
  constexpr int kOB = out_bufs(NT);
  const uint32_t ws = xs + STAGES * kXTileBytes;
  const uint32_t obuf = ws + STAGES * NT * kLrTileBytes;  // 1 KB aligned (x and low-rank tiles are)
  const uint32_t rst = obuf + kWarps * kOB * kOutTileBytes;
  const uint32_t bars = rst + max_slice_stages(NT) * 32 * 16;
  uint8_t* gbase = smem_raw + (base - smem_u32(smem_raw));
  const float4* rst_p = reinterpret_cast<const float4*>(gbase + (rst - base));
  int* cnt = reinterpret_cast<int*>(gbase + (bars - base) + 8 * STAGES);        // releases per stage
  int* issued = cnt + STAGES;                                                    // loads issued per stage
  volatile int* abort_flag = issued + STAGES;
  auto full_bar = [&](int s) { return bars + 8u * (uint32_t)s; };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int m0 = blockIdx.x * kBM;
  const int st0 = blockIdx.y * a.slice_stages;
  const int n_loc = min(a.slice_stages, a.n_stages - st0);
  const int r0 = blockIdx.z * 8 * NT;
  const int ntl = NT > 0 ? min(NT, (a.r_tot - r0) / 8) : 0;  // live low-rank tiles of this CTA
  const bool emit = blockIdx.z == 0 && (a.write_a16 || PACKED);

  auto issue = [&](int s, int c) {
    const uint32_t bar = full_bar(s);
    issued[s] += 1;
    mbar_arrive_expect_tx(bar, kXTileBytes + (uint32_t)ntl * kLrTileBytes);
    const int kx = (st0 + c) * kBK;
    tma_load_2d(xs + s * kXTileBytes, &tm_x, bar, kx, m0);
    for (int t = 0; t < ntl; ++t) {
      const int r = r0 + 8 * t;
      const uint32_t dst = ws + (s * NT + t) * kLrTileBytes;
      if (r < a.rank) tma_load_2d(dst, &tm_l2, bar, kx, r);
      else tma_load_2d(dst, &tm_lora, bar, kx, r - a.rank);
    }
  };

  if (tid == 0) {
    prefetch_tma_desc(&tm_x);
    if (ntl > 0) { prefetch_tma_desc(&tm_l2); prefetch_tma_desc(&tm_lora); }
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      cnt[s] = 0;
      issued[s] = 0;
    }
    *abort_flag = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  pdl_wait();  // inputs may come from the previous kernel on the stream
  if (tid == 0)
    for (int s = 0; s < STAGES && s < n_loc; ++s) issue(s, s);
  // reciprocal table of the slice: {RN(1/s_c), RN(1/s_c+1), -s_c, -s_c+1} per column pair.  A slice
  // with a smoothing factor outside the normal range divides with IEEE division throughout.
  bool slice_ieee;
  {
    // every load first (one round trip for the whole table), then the reciprocals
    constexpr int kTblIters = max_slice_stages(NT) * (kBK / 2) / kThreads;
    static_assert(kTblIters * kThreads == max_slice_stages(NT) * (kBK / 2), "table entries per thread");
    float4* tbl = reinterpret_cast<float4*>(gbase + (rst - base));
    float sv[kTblIters][2];
#pragma unroll
    for (int u = 0; u < kTblIters; ++u) {
      const int i = tid + u * kThreads;
      const int col = st0 * kBK + 2 * i;
      const bool live = i < n_loc * (kBK / 2);
      sv[u][0] = live && col < a.K_in ? __bfloat162float(a.smooth[col]) : 1.f;
      sv[u][1] = live && col + 1 < a.K_in ? __bfloat162float(a.smooth[col + 1]) : 1.f;
    }
    // A smoothing factor outside the normal range (zero, subnormal, inf, NaN), or in W4A4 mode below
    // 2^-64, sends the slice through IEEE division: with every |s| >= 2^-64, an x whose Markstein
    // quotient may be off (|x| < 2^-118) has |x_hat| < 2^-53, far below the smallest group scale
    // (bf16(1e-8) / 7), so it can neither be a group maximum that sets the scale nor get a nonzero
    // code, and the codes and scales stay exact without a per-element test.
    constexpr float kSmoothMin = W4A16 ? 1.17549435e-38f : 5.42101086e-20f;
    int odd_smooth = 0;
#pragma unroll
    for (int u = 0; u < kTblIters; ++u) {
      const int i = tid + u * kThreads;
      if (i < n_loc * (kBK / 2)) {
        tbl[i] = make_float4(__frcp_rn(sv[u][0]), __frcp_rn(sv[u][1]), -sv[u][0], -sv[u][1]);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float m = fabsf(sv[u][h]);
          odd_smooth |= !(m >= kSmoothMin && m <= 3.40282347e38f);
        }
      }
    }
    slice_ieee = __syncthreads_or(odd_smooth) != 0;
  }

  float acc[NT > 0 ? NT : 1][4];
#pragma unroll
  for (int t = 0; t < (NT > 0 ? NT : 1); ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f;

  const float eps = __bfloat162float(__float2bfloat16_rn(1e-8f));
  const float y7 = __frcp_rn(7.0f);
  // rint by one add: for |t| < 2^22, t + 1.5 * 2^23 rounds t to the nearest integer (ties to even)
  // and the low mantissa bits hold rint(t) in two's complement.  kMagic * scale has at most 10
  // significant bits, so fma(m, scale, -kMagic * scale) = rint(t) * scale exactly.
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  const uint64_t mag2 = f2_pack(kMagic, kMagic);
  const int wrow = warp * 16;              // first row of this warp within the CTA tile
  const int row_g = m0 + wrow + g;         // global rows held by this lane
  const int row_g8 = row_g + 8;
  const bool write_a16 = a.write_a16 != 0;
  const uint32_t cnt_base = smem_u32(cnt);
  bool ok = true;
  bool a16_range = false;  // some group scale of this lane exceeded kA16ScaleMax

  // A-fragment address of k16 block kk for this lane within a 64 x 64 swizzled tile
  const int a_row = wrow + (lane & 15);
  const int a_chk = lane >> 4;
  // B-fragment (two 8-row tiles) address offsets
  const int b_row = (lane & 7) + ((lane >> 4) << 3);
  const int b_chk = (lane >> 3) & 1;

  // k16 steps outermost so the NT accumulator chains advance side by side
  const bool all_l2 = !LORA && ntl == NT;  // every tile of this CTA is a live l2 tile (the common case)
  auto lowrank_mma = [&](const uint32_t (&fr)[4][4], int s, bool lora_pass) {
    if constexpr (NT > 0) {
      constexpr bool kF16 = W4A16;
      if (!lora_pass && all_l2) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
          for (int t = 0; t < NT; t += 2) {
            uint32_t b[4];
            ldmatrix_x4(ws + (s * NT + t) * kLrTileBytes + swz128(b_row, 2 * kk + b_chk), b);
            mma_16816<kF16>(acc[t], fr[kk], b[0], b[1]);
            mma_16816<kF16>(acc[t + 1], fr[kk], b[2], b[3]);
          }
        }
        return;
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
        for (int t = 0; t < NT; t += 2) {
          const bool l0 = t < ntl && (!LORA || ((r0 + 8 * t >= a.rank) == lora_pass));
          const bool l1 = t + 1 < ntl && (!LORA || ((r0 + 8 * (t + 1) >= a.rank) == lora_pass));
          if (!(l0 || l1)) continue;
          uint32_t b[4];
          ldmatrix_x4(ws + (s * NT + t) * kLrTileBytes + swz128(b_row, 2 * kk + b_chk), b);
          if (l0) {
            if (LORA && lora_pass) mma_16816<false>(acc[t], fr[kk], b[0], b[1]);
            else mma_16816<kF16>(acc[t], fr[kk], b[0], b[1]);
          }
          if (l1) {
            if (LORA && lora_pass) mma_16816<false>(acc[t + 1], fr[kk], b[2], b[3]);
            else mma_16816<kF16>(acc[t + 1], fr[kk], b[2], b[3]);
          }
        }
      }
    }
  };

  // lane 0: count this warp's release of stage-slot s (chunk c); the last release refills it
  auto release = [&](int s, int c) {
    const uint32_t old = atom_add_acq_rel(cnt_base + 4u * (uint32_t)s, 1u);
    if ((old & (kWarps - 1)) == kWarps - 1) {
      fence_proxy_async_smem();
      if (c + STAGES < n_loc) issue(s, c + STAGES);
    }
  };

  // x_hat of chunk c's fragments with IEEE division (__fdiv_rn), x read from global memory in
  // the fragment layout (the stage may already be refilled); rows >= M and columns >= K_in read
  // as zero, as the TMA box does.  Rare: see the exact-division note at the top of the file.
  auto ieee_chunk = [&](uint32_t (&frj)[4][4], int c) {
    const float4* tb = rst_p + c * (kBK / 2) + t4;
    const int kcol = (st0 + c) * kBK + 2 * t4;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const float4 cA = tb[8 * kk], cB = tb[8 * kk + 4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int row = (i & 1) ? row_g8 : row_g;
        const int col = kcol + 16 * kk + (i >= 2 ? 8 : 0);
        const uint32_t xr = (row < a.M && col < a.K_in)
                                ? __ldg(reinterpret_cast<const unsigned int*>(a.x + (int64_t)row * a.ldx + col))
                                : 0u;
        const float s0 = i < 2 ? -cA.z : -cB.z, s1 = i < 2 ? -cA.w : -cB.w;
        const uint64_t q = f2_pack(__fdiv_rn(__uint_as_float(xr << 16), s0),
                                   __fdiv_rn(__uint_as_float(xr & 0xFFFF0000u), s1));
        frj[kk][i] = W4A16 ? f2_to_h2(q) : f2_to_bf2(q);
      }
    }
  };
  // |x_hat| maxima of rows g (low half) and g + 8 (high half) over the group, reduced over the
  // row's four lanes (NaN if any element is NaN)
  auto group_max = [&](const uint32_t (&frg)[GS][4][4]) {
    uint32_t mx[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t m = bf2_maxabs(frg[0][0][h], frg[0][0][h + 2]);
#pragma unroll
      for (int j = 0; j < GS; ++j)
#pragma unroll
        for (int kk = (j == 0 ? 1 : 0); kk < 4; ++kk) m = bf2_maxabs(m, bf2_maxabs(frg[j][kk][h], frg[j][kk][h + 2]));
      mx[h] = m;
    }
    uint32_t both = bf2_maxabs(__byte_perm(mx[0], mx[1], 0x5410), __byte_perm(mx[0], mx[1], 0x7632));
    both = bf2_maxabs(both, __shfl_xor_sync(0xffffffffu, both, 1));
    return bf2_maxabs(both, __shfl_xor_sync(0xffffffffu, both, 2));
  };

  const uint32_t ob_base = obuf + (uint32_t)warp * (kOB * kOutTileBytes);  // this warp's a16 staging
  int n_stored = 0;  // a16 stores this warp has issued (lane 0 commits one bulk group per store)

#pragma unroll 1
  for (int c0 = 0; c0 < n_loc && ok; c0 += GS) {
    uint32_t fr[GS][4][4];  // x fragments, then x_hat fragments (bf16x2, or f16x2 in W4A16 mode)
    // ---- per chunk: load the x fragments, LoRA MMAs on raw x, x_hat = x / smooth ----
#pragma unroll
    for (int j = 0; j < GS; ++j) {
      const int c = c0 + j, s = c % STAGES;
      const uint32_t par = (uint32_t)((c / STAGES) & 1);
      if (!mbar_test(full_bar(s), par) && !mbar_wait(full_bar(s), par, abort_flag, a.err, 0x4100 + s)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) ldmatrix_x4(xs + s * kXTileBytes + swz128(a_row, 2 * kk + a_chk), fr[j][kk]);
      if constexpr (LORA) lowrank_mma(fr[j], s, true);  // LoRA down-projection on raw x
      const float4* tb = rst_p + c * (kBK / 2) + t4;
      uint32_t off_domain = 0;  // W4A16: bit 15 / 31 set where an element needs IEEE division
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const float4 cA = tb[8 * kk], cB = tb[8 * kk + 4];
        const uint64_t yA = f2_pack(cA.x, cA.y), nA = f2_pack(cA.z, cA.w);
        const uint64_t yB = f2_pack(cB.x, cB.y), nB = f2_pack(cB.z, cB.w);
        // fragment regs: 0 = (row g, cols A), 1 = (row g+8, cols A), 2 = (row g, cols B), 3 = (row g+8, cols B)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t xv = fr[j][kk][i];
          const uint64_t q = div_f2(bf2_to_f2(xv), i < 2 ? yA : yB, i < 2 ? nA : nB);
          fr[j][kk][i] = W4A16 ? f2_to_h2(q) : f2_to_bf2(q);
          if constexpr (W4A16) off_domain |= tiny_x_lanes(xv) | big_lanes<true>(fr[j][kk][i]);
        }
      }
      if (slice_ieee || (W4A16 && __any_sync(0xffffffffu, (off_domain & 0x80008000u) != 0)))
        ieee_chunk(fr[j], c);  // rare
    }
    if (!ok) break;

    // ---- W4A4: group maxima; a quotient of 2^126 or more (or inf / NaN) redoes the group ----
    uint32_t both = 0;
    if constexpr (!W4A16) {
      both = group_max(fr);
      if (!slice_ieee && __any_sync(0xffffffffu, (big_lanes<false>(both) & 0x80008000u) != 0)) {
#pragma unroll
        for (int j = 0; j < GS; ++j) ieee_chunk(fr[j], c0 + j);
        both = group_max(fr);
      }
    }
    // ---- l2 MMAs on x_hat, then the group's stages go back to the ring ----
    if (ntl > 0 && a.rank > 0 && r0 < a.rank) {
#pragma unroll
      for (int j = 0; j < GS; ++j) lowrank_mma(fr[j], (c0 + j) % STAGES, false);
    }
    __syncwarp();
    if (lane == 0) {
#pragma unroll
      for (int j = 0; j < GS; ++j) release((c0 + j) % STAGES, c0 + j);
    }
    if (!emit) continue;

    // ---- group scale of rows g and g+8 (W4A4) ----
    uint64_t sc2[2], ys2[2], ns2[2], nms2[2];  // scale, RN(1/scale), -scale, -kMagic * scale
    if constexpr (!W4A16) {
      const float am[2] = {fabsf(__uint_as_float(both << 16)), fabsf(__uint_as_float(both & 0xFFFF0000u))};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float v = fmaxf(am[h], eps);
        const float q0 = v * y7;
        const float sc = __bfloat162float(__float2bfloat16_rn(fmaf(fmaf(-q0, 7.0f, v), y7, q0)));
        const float ys = __frcp_rn(sc);
        a16_range |= sc > kA16ScaleMax;
        sc2[h] = f2_pack(sc, sc);
        ys2[h] = f2_pack(ys, ys);
        ns2[h] = f2_pack(-sc, -sc);
        nms2[h] = f2_pack(-kMagic * sc, -kMagic * sc);
        if constexpr (PACKED) {
          const int row = h ? row_g8 : row_g;
          if (t4 == 0) {
            const int grp = (st0 + c0) * kBK / a.G;
            if (row < a.M) {
              if (a.scales) a.scales[(int64_t)row * (a.K_pad / a.G) + grp] = __float2bfloat16_rn(sc);
              if (a.ascales_t) a.ascales_t[(int64_t)grp * a.lda_s + row] = sc;
            } else if (a.ascales_t && row < a.lda_s) {
              a.ascales_t[(int64_t)grp * a.lda_s + row] = 0.0f;  // the padding rows of the last band read as zero
            }
          }
        }
      }
    }

    // ---- per chunk: codes, a16 through this warp's staging tile and a TMA store ----
#pragma unroll
    for (int j = 0; j < GS; ++j) {
      const int c = c0 + j;
      const int kcol = (st0 + c) * kBK;
      const uint32_t my_tile = ob_base + (uint32_t)(n_stored % kOB) * kOutTileBytes;
      if (write_a16) {
        // the store that last used this staging tile must have read it
        if (lane == 0 && n_stored >= kOB) bulk_wait_read<kOB - 1>();
        __syncwarp();
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t o[4];
        if constexpr (W4A16) {
#pragma unroll
          for (int i = 0; i < 4; ++i) o[i] = fr[j][kk][i];
        } else {
          uint32_t nib[4], c8[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int h = i & 1;
            const uint64_t q = div_f2(bf2_to_f2(fr[j][kk][i]), ys2[h], ns2[h]);
            const uint64_t m = f2_add(q, mag2);                 // low mantissa bits = rint(q)
            o[i] = f2_to_h2(f2_fma(m, sc2[h], nms2[h]));         // rint(q) * scale, exact in fp16
            // offset-binary code q + 8 = two's-complement low nibble with its top bit flipped
            nib[i] = (((uint32_t)m & 0xFu) | (((uint32_t)(m >> 32) & 0xFu) << 4)) ^ 0x88u;
            c8[i] = ((uint32_t)m & 0xFFu) | (((uint32_t)(m >> 32) & 0xFFu) << 8);  // two int8 codes
          }
          if constexpr (PACKED) {
            if (a.packed) {
              uint8_t* prow_g = a.packed + (int64_t)row_g * (a.K_pad / 2) + (kcol + 16 * kk + 2 * t4) / 2;
              uint8_t* prow_g8 = prow_g + (int64_t)8 * (a.K_pad / 2);
              if (row_g < a.M) { prow_g[0] = (uint8_t)nib[0]; prow_g[4] = (uint8_t)nib[2]; }
              if (row_g8 < a.M) { prow_g8[0] = (uint8_t)nib[1]; prow_g8[4] = (uint8_t)nib[3]; }
            }
            if (a.codes8) {
              int8_t* crow_g = a.codes8 + (int64_t)row_g * a.K_pad + kcol + 16 * kk + 2 * t4;
              int8_t* crow_g8 = crow_g + (int64_t)8 * a.K_pad;
              if (row_g < a.M) {
                *reinterpret_cast<uint16_t*>(crow_g) = (uint16_t)c8[0];
                *reinterpret_cast<uint16_t*>(crow_g + 8) = (uint16_t)c8[2];
              }
              if (row_g8 < a.M) {
                *reinterpret_cast<uint16_t*>(crow_g8) = (uint16_t)c8[1];
                *reinterpret_cast<uint16_t*>(crow_g8 + 8) = (uint16_t)c8[3];
              }
            }
          }
        }
        if (write_a16) stmatrix_x4(my_tile + swz128(lane & 15, 2 * kk + (lane >> 4)), o[0], o[1], o[2], o[3]);
      }
      if (write_a16) {
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (m0 + wrow < a.M) tma_store_2d(&tm_a16, my_tile, kcol, m0 + wrow);
          bulk_commit();
        }
        ++n_stored;
      }
    }
  }

  pdl_trigger();  // the next kernel may start its prologue (it waits for this grid before reading)

  // ---- low-rank projection: fp32 partial of this K slice (a second launch adds the slices) ----
  if constexpr (NT > 0) {
    if (ok && a.partial) {
      float* part = a.partial + (int64_t)blockIdx.y * a.M * a.r_tot;
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        if (t < ntl) {
          const int col = r0 + 8 * t + 2 * t4;
          if (row_g < a.M)
            *reinterpret_cast<float2*>(part + (int64_t)row_g * a.r_tot + col) = make_float2(acc[t][0], acc[t][1]);
          if (row_g8 < a.M)
            *reinterpret_cast<float2*>(part + (int64_t)row_g8 * a.r_tot + col) = make_float2(acc[t][2], acc[t][3]);
        }
      }
    }
  }
  if (__any_sync(0xffffffffu, a16_range) && lane == 0 && a.write_a16) atomicCAS(a.err, 0, kErrA16Range);
  if (lane == 0) bulk_wait0();
  __syncthreads();
  if (tid == 0) {
    // no load may still be landing when the CTA exits (only possible after an abort)
    for (int s = 0; s < STAGES; ++s)
      if (issued[s] > 0 && !mbar_wait_drain(full_bar(s), (uint32_t)((issued[s] - 1) & 1), kWaitLimitNs))
        atomicCAS(a.err, 0, 0x4180 + s);
  }
}

// mid_hl[m] = [hi(v) | lo(v) | 0], v = (sum of the K-slice partials, in slice order) * column scale
// (LoRA columns), hi = bf16(v), lo = bf16(v - hi).  A thread owns four adjacent columns of one row
// (or eight padding columns) and keeps the loads of all slices in flight.  A separate launch:
// reducing in the last-arriving CTA of each row band left the work to one CTA per band at the end
// of the pass, which measured slower (38 -> 50 us at rank 32, 60 -> 103 us at rank 96).
__global__ void mid_finalize_kernel(const float* __restrict__ partial, int ksplit, int M, int rank, int r_tot,
                                    const float* __restrict__ lora_col_scale, __nv_bfloat16* __restrict__ mid_hl,
                                    int R2) {
  pdl_wait();
  pdl_trigger();
  const int c4 = r_tot / 4, p8 = (R2 - 2 * r_tot) / 8;  // value items, padding items per row
  const int w = c4 + p8;
  const int64_t total = (int64_t)M * w, kstride = (int64_t)M * r_tot / 4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(i / w), e = (int)(i % w);
    __nv_bfloat16* out = mid_hl + (int64_t)row * R2;
    if (e < c4) {
      const int j = 4 * e;
      const float4* src = reinterpret_cast<const float4*>(partial + (int64_t)row * r_tot + j);
      float4 v = __ldg(src);
      int k = 1;
      for (; k + 4 <= ksplit; k += 4) {
        float4 t[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) t[u] = __ldg(src + (k + u) * kstride);
#pragma unroll
        for (int u = 0; u < 4; ++u) { v.x += t[u].x; v.y += t[u].y; v.z += t[u].z; v.w += t[u].w; }
      }
      for (; k < ksplit; ++k) {
        const float4 t = __ldg(src + k * kstride);
        v.x += t.x; v.y += t.y; v.z += t.z; v.w += t.w;
      }
      if (j >= rank) {  // LoRA columns (lora_rank is a multiple of 8: all four or none)
        const float4 cs = *reinterpret_cast<const float4*>(lora_col_scale + (j - rank));
        v.x *= cs.x; v.y *= cs.y; v.z *= cs.z; v.w *= cs.w;
      }
      const __nv_bfloat162 h01 = __floats2bfloat162_rn(v.x, v.y), h23 = __floats2bfloat162_rn(v.z, v.w);
      const float2 f01 = __bfloat1622float2(h01), f23 = __bfloat1622float2(h23);
      const __nv_bfloat162 l01 = __floats2bfloat162_rn(v.x - f01.x, v.y - f01.y);
      const __nv_bfloat162 l23 = __floats2bfloat162_rn(v.z - f23.x, v.w - f23.y);
      *reinterpret_cast<uint2*>(out + j) = make_uint2(bf162_bits(h01), bf162_bits(h23));
      *reinterpret_cast<uint2*>(out + r_tot + j) = make_uint2(bf162_bits(l01), bf162_bits(l23));
    } else {
      *reinterpret_cast<uint4*>(out + 2 * r_tot + 8 * (e - c4)) = make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

// ---- launch geometry (shared by the workspace query and the launch) ----
struct Geometry {
  int nt, nz, slice, ksplit;
};

int pick_nt(int r_use) {
  if (r_use <= 0) return 0;
  const int tiles = r_use / 8;
  return tiles <= 2 ? 2 : tiles <= 4 ? 4 : tiles <= 8 ? 8 : tiles <= 12 ? 12 : 8;
}

// CTAs of the activation pass that fit on one SM, from its shared memory (registers never
// bind: the launch bound plans them for min_ctas(nt) CTAs, which the shared memory also allows).
int ctas_per_sm(int nt) {
  static std::atomic<int> cache[64][5];  // per device and width; concurrent fillers agree
  int dev = 0;
  cudaGetDevice(&dev);
  const int slot = nt == 0 ? 0 : nt == 2 ? 1 : nt == 4 ? 2 : nt == 8 ? 3 : 4;
  if (dev < 0 || dev >= 64) dev = 0;
  int c = cache[dev][slot].load(std::memory_order_relaxed);
  if (c == 0) {
    const uint32_t smem = slot == 0   ? aq_smem_layout_bytes<ring_stages(0), 0>()
                          : slot == 1 ? aq_smem_layout_bytes<ring_stages(2), 2>()
                          : slot == 2 ? aq_smem_layout_bytes<ring_stages(4), 4>()
                          : slot == 3 ? aq_smem_layout_bytes<ring_stages(8), 8>()
                                      : aq_smem_layout_bytes<ring_stages(12), 12>();
    int per_sm = 0, reserved = 0;
    if (cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess ||
        per_sm <= 0)
      per_sm = 233472;
    if (cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev) != cudaSuccess ||
        reserved < 0)
      reserved = 1024;
    (void)cudaGetLastError();
    const int n = per_sm / (int)(smem + (uint32_t)reserved);
    c = std::max(1, std::min(kTargetCtasPerSm, n));
    cache[dev][slot].store(c, std::memory_order_relaxed);
  }
  return c;
}

// K slices per row band: as many as one wave of CTAs holds (ctas_per_sm per SM), each slice a
// whole number of stages (a multiple of `step`: 2 for 128-column groups, so a group never
// straddles two slices), between kMinSliceStages and max_slice_stages.  Among the slice
// lengths that give the fewest waves the one that fills the most CTA slots is taken.
Geometry geometry(int M, int K_pad, int r_use, int step) {
  Geometry gm;
  gm.nt = pick_nt(r_use);
  gm.nz = gm.nt ? (r_use + 8 * gm.nt - 1) / (8 * gm.nt) : 1;
  const int n_st = K_pad / kBK;
  const int layers = ((M + cta_rows(gm.nt) - 1) / cta_rows(gm.nt)) * gm.nz;  // CTAs per K slice
  const int slots = num_sms() * ctas_per_sm(gm.nt);
  const int max_slice = max_slice_stages(gm.nt);
  int best_slice = max_slice, best_waves = 1 << 30;
  double best_fill = -1.0;
  for (int slice = kMinSliceStages; slice <= max_slice; slice += step) {
    const int ksplit = (n_st + slice - 1) / slice;
    const long long ctas = (long long)ksplit * layers;
    const int waves = (int)((ctas + slots - 1) / slots);
    const double fill = (double)ctas / ((double)waves * slots);
    if (waves < best_waves || (waves == best_waves && fill > best_fill + 1e-9)) {
      best_waves = waves;
      best_fill = fill;
      best_slice = slice;
    }
  }
  gm.slice = best_slice;
  gm.ksplit = (n_st + best_slice - 1) / best_slice;
  return gm;
}

// Workspace: the fp32 K-slice partials.  Covers both slice steps, so one size serves every group
// size and mode.
size_t workspace_bytes(int M, int K_pad, int r_tot) {
  if (r_tot <= 0 || M <= 0 || K_pad <= 0) return 0;
  const int ksplit = std::max(geometry(M, K_pad, r_tot, 1).ksplit, geometry(M, K_pad, r_tot, 2).ksplit);
  return sizeof(float) * (size_t)ksplit * (size_t)M * (size_t)r_tot;
}

struct LaunchSpec {
  CUtensorMap tm_x, tm_l2, tm_lora, tm_a16;
  AqArgs args;
  Geometry gm;
  int gs;
  bool w4a16, packed;
  const float* lora_col_scale;
  __nv_bfloat16* mid_hl;
  int R2;
};

template <int GS, int NT, bool W4A16, bool PACKED, bool LORA>
int launch_t(const LaunchSpec& L, cudaStream_t stream) {
  constexpr int STAGES = ring_stages(NT);
  constexpr uint32_t smem = aq_smem_layout_bytes<STAGES, NT>();
  auto kern = act_quant_kernel<GS, STAGES, NT, W4A16, PACKED, LORA>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return check_cuda(e, "activation pass: shared memory attribute");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((L.args.M + cta_rows(NT) - 1) / cta_rows(NT), L.gm.ksplit, L.gm.nz);
  cfg.blockDim = dim3(32 * cta_warps(NT));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, L.tm_x, L.tm_l2, L.tm_lora, L.tm_a16, L.args);
  if (e != cudaSuccess) return check_cuda(e, "activation pass launch");
  return check_launch("activation pass launch");
}

template <int GS, bool W4A16, bool PACKED, bool LORA>
int launch_nt(const LaunchSpec& L, cudaStream_t stream) {
  switch (L.gm.nt) {
    case 0: return launch_t<GS, 0, W4A16, PACKED, false>(L, stream);
    case 2: return launch_t<GS, 2, W4A16, PACKED, LORA>(L, stream);
    case 4: return launch_t<GS, 4, W4A16, PACKED, LORA>(L, stream);
    case 8: return launch_t<GS, 8, W4A16, PACKED, LORA>(L, stream);
    default: return launch_t<GS, 12, W4A16, PACKED, LORA>(L, stream);
  }
}

template <bool LORA>
int launch_l(const LaunchSpec& L, cudaStream_t stream) {
  if (L.w4a16) return launch_nt<1, true, false, LORA>(L, stream);
  if (L.gs == 1) return L.packed ? launch_nt<1, false, true, LORA>(L, stream) : launch_nt<1, false, false, LORA>(L, stream);
  return L.packed ? launch_nt<2, false, true, LORA>(L, stream) : launch_nt<2, false, false, LORA>(L, stream);
}

int launch(const LaunchSpec& L, cudaStream_t stream) {
  const int st = L.args.lora_rank > 0 ? launch_l<true>(L, stream) : launch_l<false>(L, stream);
  if (st || !L.args.partial) return st;
  const int64_t items = (int64_t)L.args.M * (L.args.r_tot / 4 + (L.R2 - 2 * L.args.r_tot) / 8);
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((items + 255) / 256, (int64_t)num_sms() * 8));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, mid_finalize_kernel, (const float*)L.args.partial, L.gm.ksplit,
                                           L.args.M, L.args.rank, L.args.r_tot, L.lora_col_scale, L.mid_hl, L.R2);
  if (e != cudaSuccess) return check_cuda(e, "activation pass finalize");
  return check_launch("activation pass finalize");
}
int validate_common(const void* x, int64_t ldx, const void* smooth, const void* l2, int rank, const void* lora_down,
                    const float* lora_col_scale, int lora_rank, int M, int K_in, int K_pad, void* out_a16,
                    void* out_mid_hl, int R2, void* workspace, size_t ws_bytes, const char* who) {
  const std::string w(who);
  auto bad = [&](const char* msg) { return set_error(SVDQ_ERR_INVALID_ARGUMENT, w + ": " + msg); };
  if (!(x && smooth)) return bad("x and smooth are required");
  if (!(M >= 0 && K_in > 0 && K_pad >= K_in)) return bad("need 0 < K_in <= K_pad");
  if (K_in % 8 != 0) return bad("K_in must be a multiple of 8 (pad smooth/l2 at load)");
  if (!(ldx >= K_in && ldx % 8 == 0)) return bad("ldx must be >= K_in and a multiple of 8");
  if (!(rank >= 0 && lora_rank >= 0 && rank % 8 == 0 && lora_rank % 8 == 0))
    return bad("rank and lora_rank must be non-negative multiples of 8");
  if (rank + lora_rank > 256) return bad("rank + lora_rank must be <= 256");
  if (rank > 0 && !l2) return bad("l2 is NULL");
  if (lora_rank > 0 && !(lora_down && lora_col_scale)) return bad("lora_down / lora_col_scale are NULL");
  const int r_tot = rank + lora_rank;
  if (out_mid_hl && !(R2 >= 2 * r_tot && R2 % 8 == 0)) return bad("R2 must be >= 2*(rank+lora_rank) and a multiple of 8");
  if ((reinterpret_cast<uintptr_t>(x) & 15u) || (reinterpret_cast<uintptr_t>(smooth) & 15u) ||
      (l2 && (reinterpret_cast<uintptr_t>(l2) & 15u)) || (lora_down && (reinterpret_cast<uintptr_t>(lora_down) & 15u)))
    return bad("x, smooth, l2, lora_down must be 16-byte aligned");
  if (K_pad % kBK != 0) return bad("K_pad must be a multiple of 64");
  if (out_a16 && (reinterpret_cast<uintptr_t>(out_a16) & 15u)) return bad("a16 must be 16-byte aligned");
  if (out_mid_hl && (reinterpret_cast<uintptr_t>(out_mid_hl) & 15u)) return bad("mid_hl must be 16-byte aligned");
  if (lora_col_scale && (reinterpret_cast<uintptr_t>(lora_col_scale) & 15u))
    return bad("lora_col_scale must be 16-byte aligned");
  if (out_mid_hl && r_tot > 0 && M > 0) {
    if (!workspace || ws_bytes < workspace_bytes(M, K_pad, r_tot))
      return bad("workspace missing or smaller than svdq_act_quant_workspace_bytes()");
    if (reinterpret_cast<uintptr_t>(workspace) & 255u) return bad("workspace must be 256-byte aligned");
  }
  return SVDQ_OK;
}

// Tensor maps and arguments of one activation pass.
int build_spec(LaunchSpec& L, const void* x, int64_t ldx, const void* smooth, const void* l2, bool l2_f16, int rank,
               const void* lora_down, const float* lora_col_scale, int lora_rank, int M, int K_in, int K_pad, int G,
               void* out_packed, void* out_scales, void* out_a16, void* out_mid_hl, int R2, void* workspace) {
  const int r_tot = rank + lora_rank;
  const bool want_mid = out_mid_hl && r_tot > 0;
  const int r_use = want_mid ? r_tot : 0;
  L.gm = geometry(M, K_pad, r_use, G == 128 ? 2 : 1);
  int st;
  if ((st = make_tma_2d(&L.tm_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, K_in, M, (uint64_t)ldx * 2, kBK,
                        cta_rows(L.gm.nt),
                        CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  L.tm_l2 = L.tm_x;
  L.tm_lora = L.tm_x;
  L.tm_a16 = L.tm_x;
  if (want_mid && rank > 0 &&
      (st = make_tma_2d(&L.tm_l2, l2_f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, l2,
                        K_in, rank, (uint64_t)K_in * 2, kBK, 8, CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if (want_mid && lora_rank > 0 &&
      (st = make_tma_2d(&L.tm_lora, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, lora_down, K_in, lora_rank, (uint64_t)K_in * 2,
                        kBK, 8, CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if (out_a16 && (st = make_tma_2d(&L.tm_a16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, out_a16, K_pad, M, (uint64_t)K_pad * 2,
                                   kBK, 16, CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  AqArgs& p = L.args;
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.ldx = ldx;
  p.M = M;
  p.K_in = K_in;
  p.K_pad = K_pad;
  p.rank = want_mid ? rank : 0;
  p.lora_rank = want_mid ? lora_rank : 0;
  p.r_tot = r_use;
  p.n_stages = K_pad / kBK;
  p.slice_stages = L.gm.slice;
  p.G = G;
  p.write_a16 = out_a16 != nullptr;
  p.smooth = static_cast<const __nv_bfloat16*>(smooth);
  p.packed = static_cast<uint8_t*>(out_packed);
  p.scales = static_cast<__nv_bfloat16*>(out_scales);
  p.codes8 = nullptr;
  p.ascales_t = nullptr;
  p.lda_s = 0;
  p.partial = want_mid ? static_cast<float*>(workspace) : nullptr;
  p.err = device_error_word();
  if (!p.err) return set_error(SVDQ_ERR_CUDA, "device error word unavailable");
  L.gs = G / kBK;
  L.lora_col_scale = lora_col_scale;
  L.mid_hl = static_cast<__nv_bfloat16*>(out_mid_hl);
  L.R2 = R2;
  return SVDQ_OK;
}

}  // namespace
}  // namespace svdq

extern "C" size_t svdq_act_quant_workspace_bytes(int M, int K_pad, int rank, int lora_rank) {
  return svdq::workspace_bytes(M, K_pad, rank + lora_rank);
}

extern "C" int svdq_act_quant(const void* x, int64_t ldx, const void* smooth, const void* l2, int rank,
                              const void* lora_down, const float* lora_col_scale, int lora_rank, int M, int K_in,
                              int K_pad, int a_group, void* out_packed, void* out_scales, void* out_a16,
                              void* out_mid_hl, int R2, void* workspace, size_t workspace_bytes,
                              cudaStream_t stream) {
  using namespace svdq;
  int st = validate_common(x, ldx, smooth, l2, rank, lora_down, lora_col_scale, lora_rank, M, K_in, K_pad, out_a16,
                           out_mid_hl, R2, workspace, workspace_bytes, "svdq_act_quant");
  if (st) return st;
  SVDQ_REQUIRE(a_group == 64 || a_group == 128, "svdq_act_quant: a_group must be 64 or 128");
  SVDQ_REQUIRE(K_pad % a_group == 0, "svdq_act_quant: K_pad must be a multiple of a_group");
  SVDQ_REQUIRE((out_packed == nullptr) == (out_scales == nullptr),
               "svdq_act_quant: packed codes and scales are emitted together");
  if (M == 0) return SVDQ_OK;
  LaunchSpec L;
  if ((st = build_spec(L, x, ldx, smooth, l2, false, rank, lora_down, lora_col_scale, lora_rank, M, K_in, K_pad,
                       a_group, out_packed, out_scales, out_a16, out_mid_hl, R2, workspace)))
    return st;
  L.w4a16 = false;
  L.packed = out_packed != nullptr;
  return launch(L, stream);
}

extern "C" int svdq_w4a16_prep(const void* x, int64_t ldx, const void* smooth, const void* l2_f16, int rank,
                               const void* lora_down, const float* lora_col_scale, int lora_rank, int M, int K_in,
                               int K_pad, void* out_a16, void* out_mid_hl, int R2, void* workspace,
                               size_t workspace_bytes, cudaStream_t stream) {
  using namespace svdq;
  int st = validate_common(x, ldx, smooth, l2_f16, rank, lora_down, lora_col_scale, lora_rank, M, K_in, K_pad,
                           out_a16, out_mid_hl, R2, workspace, workspace_bytes, "svdq_w4a16_prep");
  if (st) return st;
  SVDQ_REQUIRE(out_a16, "svdq_w4a16_prep: out_a16 is required");
  if (M == 0) return SVDQ_OK;
  LaunchSpec L;
  if ((st = build_spec(L, x, ldx, smooth, l2_f16, true, rank, lora_down, lora_col_scale, lora_rank, M, K_in, K_pad,
                       64, nullptr, nullptr, out_a16, out_mid_hl, R2, workspace)))
    return st;
  L.w4a16 = true;
  L.packed = false;
  return launch(L, stream);
}

extern "C" int svdq_act_quant_i8(const void* x, int64_t ldx, const void* smooth, const void* l2, int rank,
                                 const void* lora_down, const float* lora_col_scale, int lora_rank, int M, int K_in,
                                 int K_pad, int a_group, void* out_codes8, float* out_ascales_t, int64_t lda_s,
                                 void* out_mid_hl, int R2, void* workspace, size_t workspace_bytes,
                                 cudaStream_t stream) {
  using namespace svdq;
  int st = validate_common(x, ldx, smooth, l2, rank, lora_down, lora_col_scale, lora_rank, M, K_in, K_pad, nullptr,
                           out_mid_hl, R2, workspace, workspace_bytes, "svdq_act_quant_i8");
  if (st) return st;
  SVDQ_REQUIRE(a_group == 64 || a_group == 128, "svdq_act_quant_i8: a_group must be 64 or 128");
  SVDQ_REQUIRE(K_pad % a_group == 0, "svdq_act_quant_i8: K_pad must be a multiple of a_group");
  SVDQ_REQUIRE(out_codes8 && out_ascales_t, "svdq_act_quant_i8: codes and scales outputs are required");
  SVDQ_REQUIRE((reinterpret_cast<uintptr_t>(out_codes8) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(out_ascales_t) & 15u) == 0,
               "svdq_act_quant_i8: codes and scales must be 16-byte aligned");
  SVDQ_REQUIRE(lda_s >= M, "svdq_act_quant_i8: lda_s must be >= M");
  if (M == 0) return SVDQ_OK;
  LaunchSpec L;
  if ((st = build_spec(L, x, ldx, smooth, l2, false, rank, lora_down, lora_col_scale, lora_rank, M, K_in, K_pad,
                       a_group, nullptr, nullptr, nullptr, out_mid_hl, R2, workspace)))
    return st;
  L.args.codes8 = static_cast<int8_t*>(out_codes8);
  L.args.ascales_t = out_ascales_t;
  L.args.lda_s = lda_s;
  L.w4a16 = false;
  L.packed = true;
  return launch(L, stream);
}
