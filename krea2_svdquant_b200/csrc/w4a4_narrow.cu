// Narrow-batch W4A4 GEMM (sm_100a): up to 16 tokens against the packed INT4 weight, with the
// products on mma.sync int8 fragments held in registers.
//
// At 16 tokens the layer's arithmetic is a few GFLOP against 50 MB of weight codes (K 6144,
// N 16384): the time is the weight stream.  The tcgen05 int8-code kernel (packed_small.cu) spends
// it on the CUDA-core side: it converts the codes into shared memory for the MMA and reads each
// K group's int32 result back out of tensor memory to rescale it.  Here operands and results stay
// in registers:
//  - a warp owns 16 weight rows (two n8 tiles of mma.m16n8k32).  The codes of a CTA's 64 rows
//    arrive by TMA, two 64-row x 128-byte boxes (128-byte swizzle) per 512-wide K chunk, in a
//    two-stage ring.  Streaming them with 8-byte loads into registers measured 51 us at 16 tokens
//    (K 6144, N 16384; DRAM 14% busy, warps waiting on the loads), and with one 256-byte bulk copy
//    per row and chunk 30.7 us whatever the CTA shape: ~1,300 small copies per SM;
//  - a lane's 8 bytes of a row are the 16 nibbles k in [16 t4, 16 t4 + 16) of one 64-wide group.
//    Two mask operations turn each 32-bit word (nibble order [k0 k2 k4 k6 | k1 k3 k5 k7], as
//    svdq_prepare_packed writes it) into the two u8 B registers of one k-step, whose bytes hold
//    k = {0, 4, 1, 5} and {2, 6, 3, 7} of the word.  The activation fragments are staged with the
//    same byte order, so each MMA still sums over whole groups and the products are unchanged;
//  - the activation codes (signed int8) of each 512-wide K chunk are staged once per CTA in
//    shared memory, already in fragment order, with their group scales and 8 x their code sums;
//  - a group's int32 result d = sum a (q + 8) gives sum a q = d - 8 sum a, exact in fp32
//    (|.| <= 64 * 8 * 8), scaled by s_a * s_w into an fp32 accumulator:
//      out[m, n] = sum_g s_w[n, g] s_a[m, g] sum_{k in g} q_w[n, k] q_a[m, k]
//                + mid_hl[m] . up_hl[n] + bias[n]
//    the reference's W4A4 formula (README.md:64; the residual product of
//    src/krea2_svdquant/quant/svd.py:158 on quantized activations, low-rank up + bias of
//    svd.py:159-162), as svdq_w4a4_gemm computes it.
// The low-rank term (bf16 mma.m16n8k16 over R2) and the bias join the same accumulators.
#include "svdq_common.cuh"

namespace svdq {
namespace {

constexpr int kNwWarps = 4;
constexpr int kNwThreads = 32 * kNwWarps;
constexpr int kNwCtaRows = 16 * kNwWarps;                   // weight rows per CTA (a cluster of two)
constexpr int kNwTileRows = 128;                            // rows per tile of the scales16 layout
constexpr int kNwGroupK = 64;                               // K per group (weights and activations)
constexpr int kNwChunkGroups = 8;                           // groups per staged activation chunk
constexpr int kNwChunkK = kNwChunkGroups * kNwGroupK;       // 512
constexpr int kNwStages = 2;                                // weight ring stages per CTA
constexpr int kNwBoxBytes = kNwCtaRows * 128;               // one TMA box: the CTA's rows x 128 bytes
constexpr int kNwStageBytes = 2 * kNwBoxBytes;              // one 512-wide chunk: two 256-k halves
constexpr int kNwErrWait = 0x4401;                          // device error word: weight wait ran out

struct NarrowArgs {
  const int8_t* codes8;         // [M, K_pad] activation codes q in [-8, 7]
  const float* ascales_t;       // [K_pad / 64, lda_s] activation group scales, group-major
  int64_t lda_s;
  const uint8_t* codes;         // [N, K_pad / 2] weight codes q + 8, prepared nibble order
  const __half* scales16;       // weight group scales, prepared tile order
  const __nv_bfloat16* mid_hl;  // [M, R2]
  const __nv_bfloat16* up_hl;   // [N, R2]
  int R2;
  const __nv_bfloat16* bias;    // [N] or null
  void* out;
  int64_t ldo;
  int M, N, K_pad;
  int* err;
};

// Activation operands of two 512-wide chunks (double buffer), per 16-token tile.
template <int MT>
struct NarrowStage {
  uint4 a[2][MT][kNwChunkGroups][2][32];  // [buffer][tile][group][k-step][lane] = {a0, a1, a2, a3}
  // per token: {activation group scale, bits of the float 1.5 * 2^23 - 8 x the group's code sum}
  float2 sa[2][MT][kNwChunkGroups][16];
};

__device__ __forceinline__ void mma_s8u8(int (&d)[4], const uint4& a, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint2 lds_u2(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}
__device__ __forceinline__ float ld_dsmem_f32(uint32_t cluster_addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(cluster_addr) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ldg_u32(const __nv_bfloat16* p) {
  return __ldg(reinterpret_cast<const unsigned int*>(p));
}
// Integers |v| < 2^22 to fp32 exactly: the bits of 1.5 * 2^23 plus v are the float 1.5 * 2^23 + v.
constexpr int kMagicBits = 0x4B400000;
constexpr float kMagic = 12582912.0f;
__device__ __forceinline__ float half_bits(uint32_t w, int hi) {
  return __half2float(__ushort_as_half((unsigned short)(hi ? w >> 16 : w & 0xFFFFu)));
}

// Shared memory: the activation stage, then (1024-byte aligned, for the 128-byte swizzle) the
// weight ring, its barriers and the CTA's abort flag.
template <int MT>
__host__ __device__ constexpr uint32_t nw_smem_bytes() {
  return (uint32_t)sizeof(NarrowStage<MT>) + 1024 + kNwStages * kNwStageBytes + kNwStages * 8 + 16;
}

// Activation chunk staging, in two halves so that the loads of chunk c + 1 are in flight while
// chunk c is computed.  Item i = ((tile * 8 + group) * 16 + token) * 4 + part: 16 codes
// k in [16 part, 16 part + 16) of one group and token (the four parts of a token and group sit in
// adjacent lanes, which add their code sums by shuffles).
template <int MT>
constexpr int kNwItems = 512 * MT / kNwThreads;  // staging items per thread and chunk
template <int MT>
struct StageRegs {
  uint4 v[kNwItems<MT>];
  float as[kNwItems<MT>];
};
template <int MT>
__device__ __forceinline__ void stage_load(StageRegs<MT>& sr, int chunk, const NarrowArgs& a, int tid) {
#pragma unroll
  for (int u = 0; u < kNwItems<MT>; ++u) {
    const int i = tid + u * kNwThreads;
    const int p = i & 3, r = (i >> 2) & 15, q = (i >> 6) & 7, tt = i >> 9;
    const int m = tt * 16 + r;
    const int k0 = chunk * kNwChunkK + q * kNwGroupK + 16 * p;
    sr.v[u] = m < a.M ? __ldg(reinterpret_cast<const uint4*>(a.codes8 + (int64_t)m * a.K_pad + k0))
                      : make_uint4(0u, 0u, 0u, 0u);
    sr.as[u] = m < a.M && p == 0 ? __ldg(a.ascales_t + (int64_t)(chunk * kNwChunkGroups + q) * a.lda_s + m) : 0.0f;
  }
}
template <int MT>
__device__ __forceinline__ void stage_store(NarrowStage<MT>& sm, int buf, const StageRegs<MT>& sr, int tid) {
#pragma unroll
  for (int u = 0; u < kNwItems<MT>; ++u) {
    const int i = tid + u * kNwThreads;
    const int p = i & 3, r = (i >> 2) & 15, q = (i >> 6) & 7, tt = i >> 9;
    const uint4 v = sr.v[u];
    int s = __dp4a((int)v.x, 0x01010101, 0);
    s = __dp4a((int)v.y, 0x01010101, s);
    s = __dp4a((int)v.z, 0x01010101, s);
    s = __dp4a((int)v.w, 0x01010101, s);
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if (p == 0) sm.sa[buf][tt][q][r] = make_float2(sr.as[u], __int_as_float(kMagicBits - 8 * s));
    // lane (g, t4) = (r mod 8, p); rows 8..15 of the tile are the a1 / a3 registers
    uint32_t* d0 = reinterpret_cast<uint32_t*>(&sm.a[buf][tt][q][0][(r & 7) * 4 + p]);
    uint32_t* d1 = reinterpret_cast<uint32_t*>(&sm.a[buf][tt][q][1][(r & 7) * 4 + p]);
    const int hi = r >> 3;
    d0[hi] = __byte_perm(v.x, v.y, 0x5140);
    d0[2 + hi] = __byte_perm(v.x, v.y, 0x7362);
    d1[hi] = __byte_perm(v.z, v.w, 0x5140);
    d1[2 + hi] = __byte_perm(v.z, v.w, 0x7362);
  }
}

// A cluster of two CTAs per 64 weight rows, each over half of the K chunks; warp w owns rows
// [16 w, 16 w + 16) of the CTA's rows as n8 tiles j = 0, 1.  The second CTA hands its fp32
// partial to the first through distributed shared memory, which adds it (a fixed order:
// deterministic) and writes the output.  Four CTAs share an SM.  At 16 tokens (K 6144, N 16384)
// one 128-row CTA over all of K took 32.8 us, the K split over a pair 30.7 us, and 64-row CTAs
// (all SMs busy) also 30.7 us; the TMA ring then gave 29.1 us.  MT 16-token tiles
// (M <= 16 * MT); launched with MT = 1.
template <int MT, bool OUT_F32>
__global__ void __launch_bounds__(kNwThreads, 4)
    w4a4_narrow_kernel(const __grid_constant__ CUtensorMap tm_w, const NarrowArgs a) {
  extern __shared__ __align__(128) uint8_t nw_smem[];
  NarrowStage<MT>& sm = *reinterpret_cast<NarrowStage<MT>*>(nw_smem);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
  const uint32_t rank = cluster_ctarank();
  const int cta_row0 = (blockIdx.x >> 1) * kNwCtaRows;
  const int row0 = cta_row0 + warp * 16;
  const int tile = row0 / kNwTileRows;
  const int n_all = a.K_pad / kNwChunkK;
  const int c_begin = rank ? (n_all + 1) / 2 : 0;
  const int n_chunks = rank ? n_all - c_begin : (n_all + 1) / 2;  // this CTA's chunks c_begin + [0, n_chunks)
  const uint32_t smem0 = smem_u32(nw_smem);
  const uint32_t ring = (smem0 + (uint32_t)sizeof(NarrowStage<MT>) + 1023u) & ~1023u;
  const uint32_t bars = ring + kNwStages * kNwStageBytes;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(nw_smem + (bars - smem0) + kNwStages * 8);
  // Stage s: box h (k half) holds the CTA's rows at 128 bytes each, 16-byte pieces XOR-swizzled by
  // row mod 8 (= g for this lane's rows 16 warp + 8 j + g).  A lane's 8 bytes of group q sit in
  // piece 2 (q mod 4) + t4 / 2 of half q / 4, at byte 8 (t4 mod 2).
  const uint32_t rd = ring + (uint32_t)((warp * 16 + g) * 128 + 8 * (t4 & 1));
  // scales16 element ((tile * C4 + c4) * 128 + r) * 4 + (group within the 256-wide chunk c4); this
  // lane's output rows r = 16 warp + 8 j + 2 t4 and r + 1 come in one 16-byte load per chunk c4:
  // {r: groups 0,1 | r: 2,3 | r+1: 0,1 | r+1: 2,3}
  const int c4n = a.K_pad / 256;
  const __half* sbase = a.scales16 + (int64_t)tile * c4n * kNwTileRows * 4 + (row0 % kNwTileRows) * 4 + 8 * t4;
  auto ld_scales = [&](int c4, int j) {
    return __ldg(reinterpret_cast<const uint4*>(sbase + (int64_t)c4 * kNwTileRows * 4 + 32 * j));
  };
  auto issue = [&](int lc) {  // one thread: the CTA rows' codes of this CTA's chunk lc (512 wide)
    const int s = lc % kNwStages;
    const uint32_t bar = bars + 8u * s, dst = ring + (uint32_t)(s * kNwStageBytes);
    const int x = (c_begin + lc) * 256;
    mbar_arrive_expect_tx(bar, (uint32_t)kNwStageBytes);
    tma_load_2d(dst, &tm_w, bar, x, cta_row0);
    tma_load_2d(dst + kNwBoxBytes, &tm_w, bar, x + 128, cta_row0);
  };

  if (tid == 0) {
    *abort_flag = 0;
    prefetch_tma_desc(&tm_w);
    for (int s = 0; s < kNwStages; ++s) mbar_init(bars + 8u * s, 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait();  // the activation codes come from the previous kernel on the stream
  int issued = 0, waited = 0;  // thread 0's copies (it alone issues them, and drains them after an abort)
  if (tid == 0)
    for (; issued < kNwStages && issued < n_chunks; ++issued) issue(issued);
  if (n_chunks > 0) {
    StageRegs<MT> sr;
    stage_load<MT>(sr, c_begin, a, tid);
    stage_store<MT>(sm, 0, sr, tid);
  }
  uint4 scn[2][2];  // weight scales of the next chunk: [256-wide half][n8 tile]
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int j = 0; j < 2; ++j) scn[h][j] = n_chunks > 0 ? ld_scales(2 * c_begin + h, j) : make_uint4(0u, 0u, 0u, 0u);

  float y[MT][2][4];  // [tile][n8 tile]: {(g, 2 t4), (g, 2 t4 + 1), (g + 8, 2 t4), (g + 8, 2 t4 + 1)}
#pragma unroll
  for (int tt = 0; tt < MT; ++tt)
#pragma unroll
    for (int j = 0; j < 2; ++j) y[tt][j][0] = y[tt][j][1] = y[tt][j][2] = y[tt][j][3] = 0.0f;

  bool ok = true;
  for (int c0 = 0; c0 < n_chunks; c0 += 2) {
#pragma unroll
    for (int hc = 0; hc < 2; ++hc) {
      const int c = c0 + hc;  // this CTA's chunk index (activation buffer hc; c0 is even)
      if (c < n_chunks) {
        __syncthreads();  // chunk c's activations are staged, and every reader of the other buffer is done
        // ... and of weight stage (c - 1) mod S, which takes chunk c - 1 + S
        if (tid == 0 && ok && c >= 1 && issued < n_chunks) issue(issued++);
        StageRegs<MT> sr;
        if (c + 1 < n_chunks) stage_load<MT>(sr, c_begin + c + 1, a, tid);
        uint4 sc[2][2];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            sc[h][j] = scn[h][j];
            if (c + 1 < n_chunks) scn[h][j] = ld_scales(2 * (c_begin + c + 1) + h, j);
          }
        const int s = c % kNwStages;
        if (ok) ok = mbar_wait(bars + 8u * s, (uint32_t)((c / kNwStages) & 1), abort_flag, a.err, kNwErrWait);
        if (ok) {
          ++waited;
          const uint32_t st = rd + (uint32_t)(s * kNwStageBytes);
#pragma unroll
          for (int q = 0; q < kNwChunkGroups; ++q) {
            const uint32_t pc = st + (uint32_t)((q >> 2) * kNwBoxBytes + (((2 * (q & 3) + (t4 >> 1)) ^ g) << 4));
            const uint2 wv[2] = {lds_u2(pc), lds_u2(pc + 8 * 128)};
            uint4 af[MT][2];
            float2 sa_lo[MT], sa_hi[MT];
#pragma unroll
            for (int tt = 0; tt < MT; ++tt) {
              af[tt][0] = sm.a[hc][tt][q][0][lane];
              af[tt][1] = sm.a[hc][tt][q][1][lane];
              sa_lo[tt] = sm.sa[hc][tt][q][g];
              sa_hi[tt] = sm.sa[hc][tt][q][g + 8];
            }
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const uint32_t b00 = wv[j].x & 0x0F0F0F0Fu, b01 = (wv[j].x >> 4) & 0x0F0F0F0Fu;
              const uint32_t b10 = wv[j].y & 0x0F0F0F0Fu, b11 = (wv[j].y >> 4) & 0x0F0F0F0Fu;
              const uint4 sv = sc[q >> 2][j];
              const int gq = q & 3;
              const float ws0 = half_bits(gq < 2 ? sv.x : sv.y, gq & 1);
              const float ws1 = half_bits(gq < 2 ? sv.z : sv.w, gq & 1);
#pragma unroll
              for (int tt = 0; tt < MT; ++tt) {
                int d[4] = {0, 0, 0, 0};
                mma_s8u8(d, af[tt][0], b00, b01);
                mma_s8u8(d, af[tt][1], b10, b11);
                // (d - 8 sum a) exactly (one add to the magic bits), times s_a * s_w
                const int bl = __float_as_int(sa_lo[tt].y), bh = __float_as_int(sa_hi[tt].y);
                const float al = sa_lo[tt].x, ah = sa_hi[tt].x;
                y[tt][j][0] = fmaf(__int_as_float(d[0] + bl) - kMagic, al * ws0, y[tt][j][0]);
                y[tt][j][1] = fmaf(__int_as_float(d[1] + bl) - kMagic, al * ws1, y[tt][j][1]);
                y[tt][j][2] = fmaf(__int_as_float(d[2] + bh) - kMagic, ah * ws0, y[tt][j][2]);
                y[tt][j][3] = fmaf(__int_as_float(d[3] + bh) - kMagic, ah * ws1, y[tt][j][3]);
              }
            }
          }
        }
        if (c + 1 < n_chunks) stage_store<MT>(sm, hc ^ 1, sr, tid);
      }
    }
  }
  // after an abort: no copy may still be landing when the CTA exits
  if (tid == 0)
    for (int c = waited; c < issued; ++c)
      if (!mbar_wait_drain(bars + 8u * (c % kNwStages), (uint32_t)((c / kNwStages) & 1), kWaitLimitNs)) {
        atomicCAS(a.err, 0, kNwErrWait + 1);
        break;
      }

  // the second CTA's partial to the first, through distributed shared memory, staged over the
  // rings (idle once every warp is done with its last chunk)
  {
    float* red = reinterpret_cast<float*>(nw_smem + (ring - smem0));
    __syncthreads();
    if (rank == 1) {
#pragma unroll
      for (int tt = 0; tt < MT; ++tt)
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) red[((tt * 2 + j) * 4 + e) * kNwThreads + tid] = y[tt][j][e];
    }
    cluster_sync();
    if (rank == 0) {
      const uint32_t peer = mapa_shared(smem_u32(red), 1u);
#pragma unroll
      for (int tt = 0; tt < MT; ++tt)
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e)
            y[tt][j][e] += ld_dsmem_f32(peer + 4u * (uint32_t)(((tt * 2 + j) * 4 + e) * kNwThreads + tid));
    }
    cluster_sync();  // the peer's shared memory stays until the first CTA has read it
    ok = __syncthreads_and(ok) != 0 && !*abort_flag;
  }
  if (rank != 0 || !ok) return;

  // low-rank up-projection: y += mid_hl @ up_hl^T (bf16 operands, fp32 accumulate)
  for (int k = 0; k < a.R2; k += 16) {
    uint32_t bu[2][2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const __nv_bfloat16* up = a.up_hl + (int64_t)(row0 + 8 * j + g) * a.R2 + k + 2 * t4;
      bu[j][0] = ldg_u32(up);
      bu[j][1] = ldg_u32(up + 8);
    }
#pragma unroll
    for (int tt = 0; tt < MT; ++tt) {
      const int m0 = tt * 16 + g, m1 = m0 + 8;
      const __nv_bfloat16* md0 = a.mid_hl + (int64_t)m0 * a.R2 + k + 2 * t4;
      const __nv_bfloat16* md1 = a.mid_hl + (int64_t)m1 * a.R2 + k + 2 * t4;
      const uint32_t a0 = m0 < a.M ? ldg_u32(md0) : 0u, a2 = m0 < a.M ? ldg_u32(md0 + 8) : 0u;
      const uint32_t a1 = m1 < a.M ? ldg_u32(md1) : 0u, a3 = m1 < a.M ? ldg_u32(md1 + 8) : 0u;
#pragma unroll
      for (int j = 0; j < 2; ++j) mma_bf16(y[tt][j], a0, a1, a2, a3, bu[j][0], bu[j][1]);
    }
  }

  // bias, then rows g and g + 8 of each token tile, columns 2 t4 and 2 t4 + 1 of each n8 tile
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int n = row0 + 8 * j + 2 * t4;
    float b0 = 0.0f, b1 = 0.0f;
    if (a.bias) {
      const float2 bb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(a.bias + n));
      b0 = bb.x;
      b1 = bb.y;
    }
#pragma unroll
    for (int tt = 0; tt < MT; ++tt) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int m = tt * 16 + g + 8 * h;
        if (m < a.M) {
          const float v0 = y[tt][j][2 * h] + b0, v1 = y[tt][j][2 * h + 1] + b1;
          if constexpr (OUT_F32) {
            *reinterpret_cast<float2*>(static_cast<float*>(a.out) + (int64_t)m * a.ldo + n) = make_float2(v0, v1);
          } else {
            *reinterpret_cast<__nv_bfloat162*>(static_cast<__nv_bfloat16*>(a.out) + (int64_t)m * a.ldo + n) =
                __floats2bfloat162_rn(v0, v1);
          }
        }
      }
    }
  }
}

template <int MT, bool F32>
int launch_narrow(const cudaLaunchConfig_t& base, const CUtensorMap& tm_w, const NarrowArgs& args) {
  auto kern = w4a4_narrow_kernel<MT, F32>;
  constexpr uint32_t smem = nw_smem_bytes<MT>();
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return check_cuda(e, "svdq_w4a4_gemm_narrow: shared memory attribute");
  cudaLaunchConfig_t cfg = base;
  cfg.dynamicSmemBytes = smem;
  e = cudaLaunchKernelEx(&cfg, kern, tm_w, args);
  if (e != cudaSuccess) return check_cuda(e, "svdq_w4a4_gemm_narrow launch");
  return check_launch("svdq_w4a4_gemm_narrow");
}

}  // namespace
}  // namespace svdq

extern "C" int svdq_w4a4_gemm_narrow(const void* codes8, const float* ascales_t, int64_t lda_s, int a_group,
                                     const void* codes, const void* scales16, int w_group, const void* mid_hl,
                                     const void* up_hl, int R2, const void* bias, void* out, int out_dtype,
                                     int64_t ldo, int M, int N, int K_pad, cudaStream_t stream) {
  using namespace svdq;
  auto aligned = [](const void* p, uintptr_t n) { return (reinterpret_cast<uintptr_t>(p) & (n - 1)) == 0; };
  SVDQ_REQUIRE(codes8 && ascales_t && codes && scales16 && out, "svdq_w4a4_gemm_narrow: null operand pointer");
  SVDQ_REQUIRE(M >= 0 && M <= 16, "svdq_w4a4_gemm_narrow: M must be in [0, 16]");
  SVDQ_REQUIRE(N > 0 && N % kNwTileRows == 0, "svdq_w4a4_gemm_narrow: N must be a positive multiple of 128");
  SVDQ_REQUIRE(K_pad > 0 && K_pad % kNwChunkK == 0, "svdq_w4a4_gemm_narrow: K_pad must be a multiple of 512");
  SVDQ_REQUIRE(a_group == 64 && w_group == 64, "svdq_w4a4_gemm_narrow: a_group and w_group must be 64");
  SVDQ_REQUIRE(lda_s >= M, "svdq_w4a4_gemm_narrow: lda_s must be >= M");
  SVDQ_REQUIRE(aligned(codes8, 16) && aligned(ascales_t, 4) && aligned(codes, 16) && aligned(scales16, 16),
               "svdq_w4a4_gemm_narrow: codes8, codes and scales16 must be 16-byte aligned");
  SVDQ_REQUIRE(R2 >= 0 && R2 % 16 == 0, "svdq_w4a4_gemm_narrow: R2 must be a multiple of 16");
  SVDQ_REQUIRE(R2 == 0 || (mid_hl && up_hl && aligned(mid_hl, 4) && aligned(up_hl, 4)),
               "svdq_w4a4_gemm_narrow: mid_hl/up_hl are NULL or not 4-byte aligned");
  SVDQ_REQUIRE(!bias || aligned(bias, 4), "svdq_w4a4_gemm_narrow: bias must be 4-byte aligned");
  SVDQ_REQUIRE(out_dtype == SVDQ_BF16 || out_dtype == SVDQ_FP32,
               "svdq_w4a4_gemm_narrow: out_dtype must be bf16 or fp32");
  SVDQ_REQUIRE(ldo >= N && ldo % 2 == 0 && aligned(out, out_dtype == SVDQ_FP32 ? 8 : 4),
               "svdq_w4a4_gemm_narrow: ldo must be even and >= N, out aligned to two elements");
  if (M == 0) return SVDQ_OK;
  NarrowArgs args;
  args.codes8 = static_cast<const int8_t*>(codes8);
  args.ascales_t = ascales_t;
  args.lda_s = lda_s;
  args.codes = static_cast<const uint8_t*>(codes);
  args.scales16 = static_cast<const __half*>(scales16);
  args.mid_hl = static_cast<const __nv_bfloat16*>(mid_hl);
  args.up_hl = static_cast<const __nv_bfloat16*>(up_hl);
  args.R2 = R2;
  args.bias = static_cast<const __nv_bfloat16*>(bias);
  args.out = out;
  args.ldo = ldo;
  args.M = M;
  args.N = N;
  args.K_pad = K_pad;
  args.err = device_error_word();
  if (!args.err) return set_error(SVDQ_ERR_CUDA, "svdq_w4a4_gemm_narrow: device error word unavailable");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * (N / kNwCtaRows));
  cfg.blockDim = dim3(kNwThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 2;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const bool f32 = out_dtype == SVDQ_FP32;
  CUtensorMap tm_w;  // the codes as [N rows][K_pad / 2 bytes], 64-row x 128-byte boxes
  const int st = make_tma_2d(&tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, codes, (uint64_t)K_pad / 2, (uint64_t)N,
                             (uint64_t)K_pad / 2, 128, kNwCtaRows, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  return f32 ? launch_narrow<1, true>(cfg, tm_w, args) : launch_narrow<1, false>(cfg, tm_w, args);
}
