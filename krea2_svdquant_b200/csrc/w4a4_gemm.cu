// Fused W4A4 SVDQuant GEMM for sm_100a (tcgen05 + TMA + TMEM).
//
//   out[m, n] = sum_g sa[m,g] sw[n,g] P_g[m,n] + sum_j mid_hl[m,j] up_hl[n,j] + bias[n]
//   P_g[m,n]  = sum_{k in 64-group g} qa[m,k] qw[n,k]       (integers, |P_g| <= 4096)
//
// Persistent kernel, one 128x256 output tile at a time per CTA, 12 warps:
//   warp 0      TMA producer: per stage one 128-byte K slice of A (codes or
//               mid_hl) and B (codes or up_hl) with 128B swizzle, plus the
//               two 64-groups' scale rows (sa^T, sw^T) of that slice.
//   warp 1      TMEM allocator and MMA issuer.  Each 64-group is two
//               kind::f8f6f4 MMAs (e4m3 codes hold the integers exactly, the
//               fp32 partial P_g is exact) into one of two 256-column TMEM
//               buffers; the low-rank/LoRA term is kind::f16 MMAs over
//               mid_hl x up_hl into a buffer of its own.
//   warps 4-11  rescale + epilogue: two warpgroups, each owning 128 of the
//               256 columns of the 128 TMEM lanes.  They drain a buffer with
//               tcgen05.ld (16x256b shape, double-buffered), free it for the
//               next group, and fold it into fp32 register accumulators with
//               packed f32x2 math: acc += P_g * (sa * sw).  After the last
//               group: + bias, cast, store.
// Every wait is bounded; a wait that runs out sets a CTA abort flag and the
// library's device error word, and all roles leave their loops.
#include "svdq_common.cuh"

namespace svdq {
namespace {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int KB = 128;  // bytes of K per stage row (two 64-groups of e4m3, or 64 bf16)
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * KB;
constexpr int B_BYTES = BN * KB;
constexpr int SA_BYTES = 2 * BM * 4;
constexpr int SW_BYTES = 2 * BN * 4;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SA_BYTES + SW_BYTES;  // 51 KiB, 1 KiB multiple
constexpr int NUM_THREADS = 384;
constexpr int TMEM_COLS = 512;  // two 256-column fp32 accumulators
constexpr int EPI_COLS = 128;   // columns per rescale warpgroup
// Register split: 384 threads launch with 168 registers each (64512); the
// producer/MMA warpgroup drops to 40 and the two rescale warpgroups rise to 232
// (128*40 + 256*232 = 64512).  The host refuses to launch if the compiled
// kernel's register count differs, since the split would then not balance.
constexpr int LAUNCH_REGS = 168;
constexpr int REGS_CTRL = 40;
constexpr int REGS_EPI = 232;
static_assert(128 * REGS_CTRL + 256 * REGS_EPI == NUM_THREADS * LAUNCH_REGS, "register split");

static_assert(STAGE_BYTES % 1024 == 0, "stage must keep 1 KiB alignment for 128B swizzle");

struct Barriers {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
};

constexpr size_t SMEM_BYTES = (size_t)STAGES * STAGE_BYTES + sizeof(Barriers) + 1024;

struct GemmArgs {
  const __nv_bfloat16* bias;
  void* out;
  int64_t ldo;
  int M, N;
  int n_groups;  // K_pad / 64
  int n_lr;      // R2 / 64 low-rank stages
  int num_m_blocks, num_n_blocks;
  int* err;
};

// Wait sites recorded in the device error word.
enum : int {
  kWaitProdEmpty = 0x101,
  kWaitMmaFull = 0x201,
  kWaitMmaTmemEmpty = 0x202,
  kWaitMmaDone = 0x203,
  kWaitEpiTmemFull = 0x301,
  kWaitEpiFull = 0x302,
};

__device__ __forceinline__ void advance(int& stage, uint32_t& phase, int n) {
  if (++stage == n) {
    stage = 0;
    phase ^= 1u;
  }
}

template <bool OUT_F32>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    w4a4_gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                     const __grid_constant__ CUtensorMap tm_sa, const __grid_constant__ CUtensorMap tm_sw,
                     const __grid_constant__ CUtensorMap tm_mid, const __grid_constant__ CUtensorMap tm_up,
                     const GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw_addr & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  const uint32_t smem_base = raw_addr + pad;
  Barriers* bars = reinterpret_cast<Barriers*>(smem + (size_t)STAGES * STAGE_BYTES);
  volatile int* abort_flag = &bars->abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_ks = (args.n_groups + 1) / 2;  // K stages (two groups each; last may hold one)
  const int num_tiles = args.num_m_blocks * args.num_n_blocks;

  auto full_bar = [&](int s) { return smem_u32(&bars->full[s]); };
  auto empty_bar = [&](int s) { return smem_u32(&bars->empty[s]); };
  auto stage_a = [&](int s) { return smem_base + (uint32_t)(s * STAGE_BYTES); };
  auto stage_b = [&](int s) { return smem_base + (uint32_t)(s * STAGE_BYTES + A_BYTES); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1 + 8);  // MMA commit + one arrival per rescale warp
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&bars->tmem_full[b]), 1);
      mbar_init(smem_u32(&bars->tmem_empty[b]), 8);
    }
    mbar_init(smem_u32(&bars->mma_done), 1);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tma_desc(&tm_a);
    prefetch_tma_desc(&tm_b);
    prefetch_tma_desc(&tm_sa);
    prefetch_tma_desc(&tm_sw);
    if (args.n_lr > 0) {
      prefetch_tma_desc(&tm_mid);
      prefetch_tma_desc(&tm_up);
    }
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&bars->tmem_base), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;

  if (warp < 4) {
    setmaxnreg_dec<REGS_CTRL>();
    if (warp == 0) {
      // ------------------------------------------------------------ producer
      if (lane == 0) {
        int stage = 0;
        uint32_t phase = 0;
        uint32_t filled_mask = 0, fill_parity = 0;
        bool ok = true;
        for (int t = blockIdx.x; ok && t < num_tiles; t += gridDim.x) {
          const int m0 = (t % args.num_m_blocks) * BM;
          const int n0 = (t / args.num_m_blocks) * BN;
          for (int j = 0; ok && j < args.n_lr; ++j) {
            if (!(ok = mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag, args.err, kWaitProdEmpty))) break;
            mbar_arrive_expect_tx(full_bar(stage), A_BYTES + B_BYTES);
            tma_load_2d(stage_a(stage), &tm_mid, full_bar(stage), j * 64, m0);
            tma_load_2d(stage_b(stage), &tm_up, full_bar(stage), j * 64, n0);
            filled_mask |= 1u << stage;
            fill_parity = (fill_parity & ~(1u << stage)) | (phase << stage);
            advance(stage, phase, STAGES);
          }
          for (int s = 0; ok && s < n_ks; ++s) {
            if (!(ok = mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag, args.err, kWaitProdEmpty))) break;
            mbar_arrive_expect_tx(full_bar(stage), STAGE_BYTES);
            tma_load_2d(stage_a(stage), &tm_a, full_bar(stage), s * KB, m0);
            tma_load_2d(stage_b(stage), &tm_b, full_bar(stage), s * KB, n0);
            tma_load_2d(stage_b(stage) + B_BYTES, &tm_sa, full_bar(stage), m0, 2 * s);
            tma_load_2d(stage_b(stage) + B_BYTES + SA_BYTES, &tm_sw, full_bar(stage), n0, 2 * s);
            filled_mask |= 1u << stage;
            fill_parity = (fill_parity & ~(1u << stage)) | (phase << stage);
            advance(stage, phase, STAGES);
          }
        }
        if (!ok) {
          // let copies already in flight land before the CTA exits
          for (int s = 0; s < STAGES; ++s)
            if (filled_mask & (1u << s)) mbar_wait_drain(full_bar(s), (fill_parity >> s) & 1u, 100000000ull);
        }
      }
    } else if (warp == 1) {
      // ------------------------------------------------------------ MMA issuer
      if (lane == 0) {
        const uint32_t idesc_bf16 = make_idesc(kFmtBF16, kFmtBF16, BM, BN);
        const uint32_t idesc_e4m3 = make_idesc(kFmtE4M3, kFmtE4M3, BM, BN);
        int stage = 0;
        uint32_t phase = 0;
        int tb = 0;
        uint32_t tphase = 0;
        bool ok = true;
        for (int t = blockIdx.x; ok && t < num_tiles; t += gridDim.x) {
          if (args.n_lr > 0) {
            if (!(ok = mbar_wait(smem_u32(&bars->tmem_empty[tb]), tphase ^ 1u, abort_flag, args.err,
                                 kWaitMmaTmemEmpty)))
              break;
            tc_fence_after();
            const uint32_t d = tmem_base + (uint32_t)(tb * BN);
            for (int j = 0; ok && j < args.n_lr; ++j) {
              if (!(ok = mbar_wait(full_bar(stage), phase, abort_flag, args.err, kWaitMmaFull))) break;
              tc_fence_after();
              const uint64_t da = desc_k_sw128(stage_a(stage));
              const uint64_t db = desc_k_sw128(stage_b(stage));
  #pragma unroll
              for (int kk = 0; kk < 4; ++kk)  // 4 x K=16 bf16 = 128 bytes
                umma_f16(d, da + (uint64_t)(kk * 2), db + (uint64_t)(kk * 2), idesc_bf16,
                         (j > 0 || kk > 0) ? 1u : 0u);
              umma_commit(empty_bar(stage));
              advance(stage, phase, STAGES);
            }
            if (!ok) break;
            umma_commit(smem_u32(&bars->tmem_full[tb]));
            advance(tb, tphase, 2);
          }
          for (int s = 0; ok && s < n_ks; ++s) {
            if (!(ok = mbar_wait(full_bar(stage), phase, abort_flag, args.err, kWaitMmaFull))) break;
            tc_fence_after();
            const uint64_t da = desc_k_sw128(stage_a(stage));
            const uint64_t db = desc_k_sw128(stage_b(stage));
            const int ngs = min(2, args.n_groups - 2 * s);
            for (int h = 0; h < ngs; ++h) {
              if (!(ok = mbar_wait(smem_u32(&bars->tmem_empty[tb]), tphase ^ 1u, abort_flag, args.err,
                                   kWaitMmaTmemEmpty)))
                break;
              tc_fence_after();
              const uint32_t d = tmem_base + (uint32_t)(tb * BN);
  #pragma unroll
              for (int kk = 0; kk < 2; ++kk) {  // 2 x K=32 e4m3 = one 64-group
                const uint64_t off = (uint64_t)((h * 64 + kk * 32) >> 4);
                umma_f8f6f4(d, da + off, db + off, idesc_e4m3, kk > 0 ? 1u : 0u);
              }
              umma_commit(smem_u32(&bars->tmem_full[tb]));
              advance(tb, tphase, 2);
            }
            if (!ok) break;
            umma_commit(empty_bar(stage));
            advance(stage, phase, STAGES);
          }
        }
        // all issued MMAs must finish before TMEM is released
        umma_commit(smem_u32(&bars->mma_done));
        if (!mbar_wait_drain(smem_u32(&bars->mma_done), 0, 1000000000ull)) {
          *abort_flag = 1;
          atomicCAS(args.err, 0, kWaitMmaDone);
        }
      }
    }
  } else {
    setmaxnreg_inc<REGS_EPI>();
    // ------------------------------------------------------------ rescale + epilogue
    // TMEM is drained with the 16x256b shape: thread i of a warp owns rows
    // {r0, r0+8, r0+16, r0+24} (r0 = 32q + i/4) and column pairs
    // {8j + 2(i%4), +1 : j = 0..15} of its warpgroup's 128 columns, so per group
    // it needs 4 activation scales and 16 weight-scale pairs.
    const int ew = warp - 4;
    const int q = warp & 3;                 // TMEM lane quarter this warp may access
    const int col0 = (ew >> 2) * EPI_COLS;  // warpgroup's column half
    const int r0 = q * 32 + (lane >> 2);
    const int cpair = 2 * (lane & 3);
    int stage = 0;
    uint32_t phase = 0;
    int tb = 0;
    uint32_t tphase = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < num_tiles; t += gridDim.x) {
      const int m0 = (t % args.num_m_blocks) * BM;
      const int n0 = (t / args.num_m_blocks) * BN;
      uint64_t acc[4][16];  // [row r0 + 8*k][column pair j]
      if (args.n_lr > 0) {
        if (!(ok = mbar_wait(smem_u32(&bars->tmem_full[tb]), tphase, abort_flag, args.err, kWaitEpiTmemFull)))
          break;
        tc_fence_after();
#pragma unroll
        for (int lh = 0; lh < 2; ++lh) {
#pragma unroll
          for (int cb = 0; cb < 2; ++cb) {
            uint32_t r[32];
            tmem_ld_16x256b_x8(tmem_base + ((uint32_t)(q * 32 + lh * 16) << 16) + (uint32_t)(tb * BN + col0 + cb * 64), r);
            tmem_ld_wait_regs(r);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              acc[2 * lh][cb * 8 + j] = ((uint64_t)r[4 * j + 1] << 32) | r[4 * j];
              acc[2 * lh + 1][cb * 8 + j] = ((uint64_t)r[4 * j + 3] << 32) | r[4 * j + 2];
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&bars->tmem_empty[tb]));
        advance(tb, tphase, 2);
        for (int j = 0; j < args.n_lr; ++j) {
          if (lane == 0) mbar_arrive(empty_bar(stage));
          advance(stage, phase, STAGES);
        }
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[k][j] = 0ull;
      }
      for (int s = 0; ok && s < n_ks; ++s) {
        if (!(ok = mbar_wait(full_bar(stage), phase, abort_flag, args.err, kWaitEpiFull))) break;
        const float* sa_s = reinterpret_cast<const float*>(smem + (size_t)stage * STAGE_BYTES + A_BYTES + B_BYTES);
        const float* sw_s = sa_s + 2 * BM;
        const int ngs = min(2, args.n_groups - 2 * s);
        for (int h = 0; h < ngs; ++h) {
          if (!(ok = mbar_wait(smem_u32(&bars->tmem_full[tb]), tphase, abort_flag, args.err, kWaitEpiTmemFull)))
            break;
          tc_fence_after();
          const float* sar = sa_s + h * BM + r0;
          uint64_t sa2[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float v = sar[8 * k];
            sa2[k] = f2_pack(v, v);
          }
          const float* swr = sw_s + h * BN + col0 + cpair;
          const uint32_t tcol = tmem_base + (uint32_t)(tb * BN + col0);
          // chunks: (cb, lh) = (0,0) (0,1) (1,0) (1,1); each 16 lanes x 64 columns.
          uint32_t pa[32], pb[32];
          tmem_ld_16x256b_x8(tcol + ((uint32_t)(q * 32) << 16), pa);
          tmem_ld_wait_regs(pa);
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) {
            const int cb = ch >> 1, lh = ch & 1;
            uint32_t (&cur)[32] = (ch & 1) ? pb : pa;
            uint32_t (&nxt)[32] = (ch & 1) ? pa : pb;
            if (ch + 1 < 4) {
              const int ncb = (ch + 1) >> 1, nlh = (ch + 1) & 1;
              tmem_ld_16x256b_x8(tcol + ((uint32_t)(q * 32 + nlh * 16) << 16) + (uint32_t)(ncb * 64), nxt);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint64_t w2 = *reinterpret_cast<const uint64_t*>(swr + (cb * 8 + j) * 8);
              const uint64_t s_lo = f2_mul(w2, sa2[2 * lh]);
              const uint64_t s_hi = f2_mul(w2, sa2[2 * lh + 1]);
              const uint64_t p_lo = ((uint64_t)cur[4 * j + 1] << 32) | cur[4 * j];
              const uint64_t p_hi = ((uint64_t)cur[4 * j + 3] << 32) | cur[4 * j + 2];
              acc[2 * lh][cb * 8 + j] = f2_fma(p_lo, s_lo, acc[2 * lh][cb * 8 + j]);
              acc[2 * lh + 1][cb * 8 + j] = f2_fma(p_hi, s_hi, acc[2 * lh + 1][cb * 8 + j]);
            }
            if (ch + 1 < 4) {
              tmem_ld_wait_regs(nxt);
              if (ch + 2 == 4) {
                // last chunk is in registers: release the TMEM buffer to the MMA warp
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&bars->tmem_empty[tb]));
              }
            }
          }
          advance(tb, tphase, 2);
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_bar(stage));
        advance(stage, phase, STAGES);
      }
      if (!ok) break;
      // epilogue: + bias, cast, store (4 rows x 16 column pairs per thread)
      float2 bias2[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int n = n0 + col0 + 8 * j + cpair;
        bias2[j] = (args.bias && n < args.N)
                       ? __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(args.bias + n))
                       : make_float2(0.f, 0.f);
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int grow = m0 + r0 + 8 * k;
        if (grow < args.M) {
          const int64_t rbase = (int64_t)grow * args.ldo;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int n = n0 + col0 + 8 * j + cpair;
            if (n < args.N) {
              const float v0 = f2_lo(acc[k][j]) + bias2[j].x;
              const float v1 = f2_hi(acc[k][j]) + bias2[j].y;
              if constexpr (OUT_F32) {
                *reinterpret_cast<float2*>(static_cast<float*>(args.out) + rbase + n) = make_float2(v0, v1);
              } else {
                *reinterpret_cast<__nv_bfloat162*>(static_cast<__nv_bfloat16*>(args.out) + rbase + n) =
                    __floats2bfloat162_rn(v0, v1);
              }
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace
}  // namespace svdq

extern "C" int svdq_w4a4_gemm(const void* act_codes, const float* act_scales_t, int ld_ast,
                              const void* w_codes, const float* w_scales_t, const void* mid_hl,
                              const void* up_hl, int R2, const void* bias, void* out, int out_dtype,
                              int64_t ldo, int M, int N, int K_pad, cudaStream_t stream) {
  using namespace svdq;
  SVDQ_REQUIRE(act_codes && act_scales_t && w_codes && w_scales_t && out,
               "svdq_w4a4_gemm: null operand pointer");
  SVDQ_REQUIRE(M >= 0 && N > 0 && K_pad > 0, "svdq_w4a4_gemm: bad M/N/K_pad");
  SVDQ_REQUIRE(K_pad % 64 == 0, "svdq_w4a4_gemm: K_pad must be a multiple of 64");
  SVDQ_REQUIRE(N % 8 == 0 && ldo >= N && ldo % 8 == 0, "svdq_w4a4_gemm: N and ldo must be multiples of 8, ldo >= N");
  SVDQ_REQUIRE(ld_ast >= M && ld_ast % 4 == 0, "svdq_w4a4_gemm: ld_ast must be >= M and a multiple of 4");
  SVDQ_REQUIRE(R2 >= 0 && R2 % 64 == 0, "svdq_w4a4_gemm: R2 must be a multiple of 64");
  SVDQ_REQUIRE(R2 == 0 || (mid_hl && up_hl), "svdq_w4a4_gemm: mid_hl/up_hl are NULL");
  SVDQ_REQUIRE(out_dtype == SVDQ_BF16 || out_dtype == SVDQ_FP32, "svdq_w4a4_gemm: out_dtype must be bf16 or fp32");
  SVDQ_REQUIRE(!bias || (reinterpret_cast<uintptr_t>(bias) & 15u) == 0, "svdq_w4a4_gemm: bias must be 16-byte aligned");
  SVDQ_REQUIRE((reinterpret_cast<uintptr_t>(out) & 15u) == 0, "svdq_w4a4_gemm: out must be 16-byte aligned");
  if (M == 0) return SVDQ_OK;
  int* err = device_error_word();
  if (!err) return set_error(SVDQ_ERR_CUDA, "svdq_w4a4_gemm: device error word unavailable");

  const int n_groups = K_pad / 64;
  CUtensorMap tm_a, tm_b, tm_sa, tm_sw, tm_mid, tm_up;
  int st;
  if ((st = make_tma_2d(&tm_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, act_codes, K_pad, M, K_pad, KB, BM,
                        CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if ((st = make_tma_2d(&tm_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, w_codes, K_pad, N, K_pad, KB, BN,
                        CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if ((st = make_tma_2d(&tm_sa, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, act_scales_t, M, n_groups,
                        (uint64_t)ld_ast * 4, BM, 2, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return st;
  if ((st = make_tma_2d(&tm_sw, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w_scales_t, N, n_groups,
                        (uint64_t)N * 4, BN, 2, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return st;
  if (R2 > 0) {
    if ((st = make_tma_2d(&tm_mid, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, mid_hl, R2, M, (uint64_t)R2 * 2,
                          64, BM, CU_TENSOR_MAP_SWIZZLE_128B)))
      return st;
    if ((st = make_tma_2d(&tm_up, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, up_hl, R2, N, (uint64_t)R2 * 2,
                          64, BN, CU_TENSOR_MAP_SWIZZLE_128B)))
      return st;
  } else {
    tm_mid = tm_a;
    tm_up = tm_b;
  }

  GemmArgs a;
  a.bias = static_cast<const __nv_bfloat16*>(bias);
  a.out = out;
  a.ldo = ldo;
  a.M = M;
  a.N = N;
  a.n_groups = n_groups;
  a.n_lr = R2 / 64;
  a.num_m_blocks = (M + BM - 1) / BM;
  a.num_n_blocks = (N + BN - 1) / BN;
  a.err = err;
  {
    cudaFuncAttributes fa;
    cudaError_t e = out_dtype == SVDQ_FP32 ? cudaFuncGetAttributes(&fa, w4a4_gemm_kernel<true>)
                                           : cudaFuncGetAttributes(&fa, w4a4_gemm_kernel<false>);
    if (e != cudaSuccess) return check_cuda(e, "svdq_w4a4_gemm: kernel attributes");
    if (fa.numRegs != LAUNCH_REGS)
      return set_error(SVDQ_ERR_UNSUPPORTED, "svdq_w4a4_gemm: kernel compiled with " + std::to_string(fa.numRegs) +
                                                 " registers/thread; the warp-group register split needs " +
                                                 std::to_string(LAUNCH_REGS));
  }
  const int tiles = a.num_m_blocks * a.num_n_blocks;
  const int grid = tiles < num_sms() ? tiles : num_sms();
  if (out_dtype == SVDQ_FP32) {
    cudaFuncSetAttribute(w4a4_gemm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
    w4a4_gemm_kernel<true><<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(tm_a, tm_b, tm_sa, tm_sw, tm_mid, tm_up, a);
  } else {
    cudaFuncSetAttribute(w4a4_gemm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
    w4a4_gemm_kernel<false><<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(tm_a, tm_b, tm_sa, tm_sw, tm_mid, tm_up, a);
  }
  return check_launch("svdq_w4a4_gemm launch");
}
