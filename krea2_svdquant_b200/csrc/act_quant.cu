// Activation quantization pass of the W4A4 SVDQuant linear (sm_100a).
//
// One pass over x [M, K_in] bf16 produces, per 16-row band:
//   x_hat = bf16(x / smooth)                             (svd.py:122)
//   q     = clamp(rint(x_hat / scale), -8, 7) per group  (pack.py:6-23)
//   scale = bf16(max(amax, bf16(1e-8)) / 7)              (pack.py:20)
//   packed nibbles (q + 8, even k low)                   (pack.py:47-56)
//   e4m3 codes (exact integers) + fp32 scales^T for the GEMM
//   mid = [x_hat @ l2^T | (x @ lora_down^T) * col_scale] (svd.py:159, linear.py:45)
//         written as a bf16 hi/lo pair so the GEMM's bf16 MMA keeps ~16 mantissa bits.
// The down-projection runs on mma.sync tensor cores from shared memory.
#include <cuda_fp8.h>

#include "svdq_common.cuh"

namespace svdq {
namespace {

constexpr int kBM = 16;        // rows per CTA
constexpr int kThreads = 128;  // 4 warps
constexpr int kStages = 3;
constexpr int kMaxTilesPerWarp = 8;  // r_tot <= 4 warps * 8 tiles * 8 cols = 256

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                            uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

struct ActQuantParams {
  const __nv_bfloat16* x;
  int64_t ldx;
  const __nv_bfloat16* smooth;
  const __nv_bfloat16* l2;     // [rank, K_in]
  const __nv_bfloat16* lora;   // [lora_rank, K_in]
  const float* lora_col_scale; // [lora_rank]
  int rank, lora_rank;
  int M, K_in, K_pad;
  uint8_t* packed;             // [M, K_pad/2]
  __nv_bfloat16* scales;       // [M, K_pad/G]
  uint8_t* codes;              // [M, K_pad] e4m3
  float* scales_t;             // [K_pad/64, ld_ast]
  int ld_ast;
  __nv_bfloat16* mid_hl;       // [M, R2]
  int R2;
};

// Shared-memory rows are padded by 8 bf16 so ldmatrix row addresses hit distinct banks.
template <int G>
struct Smem {
  static constexpr int LD = G + 8;
};

template <int G>
__global__ void __launch_bounds__(kThreads) act_quant_kernel(const ActQuantParams p) {
  constexpr int LD = Smem<G>::LD;
  constexpr int EPT = G / 8;  // elements per thread in the quant step (8 threads per row)
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int r_tot = p.rank + p.lora_rank;
  // layout: xs[kStages][kBM][LD], ws[kStages][r_tot][LD], sm[kStages][G], xh[kBM][LD]
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  __nv_bfloat16* ws = xs + kStages * kBM * LD;
  __nv_bfloat16* sm = ws + kStages * r_tot * LD;
  __nv_bfloat16* xh = sm + kStages * G;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int m0 = blockIdx.x * kBM;
  const int n_chunks = p.K_pad / G;

  // ---- async loads of one K chunk (x band, smooth slice, weight rows) ----
  auto load_chunk = [&](int c) {
    const int st = c % kStages;
    const int k0 = c * G;
    constexpr int SEG = G / 8;  // 16-byte segments per row
    // x band: kBM rows x SEG segments
    for (int i = tid; i < kBM * SEG; i += kThreads) {
      const int r = i / SEG, s = i % SEG;
      const int col = k0 + s * 8;
      const int row = m0 + r;
      int bytes = 0;
      const __nv_bfloat16* src = p.x;
      if (row < p.M && col < p.K_in) {
        bytes = min(16, (p.K_in - col) * 2);
        src = p.x + (int64_t)row * p.ldx + col;
      }
      cp_async16(smem_u32(xs + (st * kBM + r) * LD + s * 8), src, bytes);
    }
    // smooth slice (G values); padded columns read as 1 through bytes == 0 -> handled below
    for (int s = tid; s < SEG; s += kThreads) {
      const int col = k0 + s * 8;
      int bytes = 0;
      const __nv_bfloat16* src = p.smooth;
      if (col < p.K_in) {
        bytes = min(16, (p.K_in - col) * 2);
        src = p.smooth + col;
      }
      cp_async16(smem_u32(sm + st * G + s * 8), src, bytes);
    }
    // weight rows: l2 rows then lora rows
    for (int i = tid; i < r_tot * SEG; i += kThreads) {
      const int r = i / SEG, s = i % SEG;
      const int col = k0 + s * 8;
      const __nv_bfloat16* base = r < p.rank ? p.l2 + (int64_t)r * p.K_in
                                             : p.lora + (int64_t)(r - p.rank) * p.K_in;
      int bytes = 0;
      const __nv_bfloat16* src = base;
      if (col < p.K_in) {
        bytes = min(16, (p.K_in - col) * 2);
        src = base + col;
      }
      cp_async16(smem_u32(ws + (st * r_tot + r) * LD + s * 8), src, bytes);
    }
  };

  float acc[kMaxTilesPerWarp][4];
#pragma unroll
  for (int j = 0; j < kMaxTilesPerWarp; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  const int n_tiles = r_tot / 8;

  const float eps = __bfloat162float(__float2bfloat16_rn(1e-8f));
  const int qrow = tid / 8;               // quant step: row of the band
  const int qcol = (tid % 8) * EPT;       // first column of this thread within the chunk
  const int grow = m0 + qrow;

#pragma unroll 1
  for (int c = 0; c < kStages - 1; ++c) {
    if (c < n_chunks) load_chunk(c);
    cp_async_commit();
  }

#pragma unroll 1
  for (int c = 0; c < n_chunks; ++c) {
    const int st = c % kStages;
    cp_async_wait<kStages - 2>();
    __syncthreads();  // chunk c landed; everyone finished chunk c-1
    if (c + kStages - 1 < n_chunks) load_chunk(c + kStages - 1);
    cp_async_commit();

    const int k0 = c * G;
    // ---- smoothing + group quantization (bit-exact with the reference) ----
    {
      const __nv_bfloat16* xr = xs + (st * kBM + qrow) * LD + qcol;
      const __nv_bfloat16* sr = sm + st * G + qcol;
      float xhv[EPT];
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < EPT; ++i) {
        const int col = k0 + qcol + i;
        float v = 0.f;
        if (col < p.K_in) v = __bfloat162float(__float2bfloat16_rn(
                              __fdiv_rn(__bfloat162float(xr[i]), __bfloat162float(sr[i]))));
        xhv[i] = v;
        amax = fmaxf(amax, fabsf(v));
      }
#pragma unroll
      for (int i = 0; i < EPT; i += 2) {
        __nv_bfloat162 pr;
        pr.x = __float2bfloat16_rn(xhv[i]);
        pr.y = __float2bfloat16_rn(xhv[i + 1]);
        *reinterpret_cast<__nv_bfloat162*>(xh + qrow * LD + qcol + i) = pr;
      }
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
      const float scale = __bfloat162float(__float2bfloat16_rn(__fdiv_rn(fmaxf(amax, eps), 7.0f)));
      uint32_t nib[EPT / 8];
      uint32_t e4[EPT / 4];
#pragma unroll
      for (int i = 0; i < EPT / 8; ++i) nib[i] = 0;
#pragma unroll
      for (int i = 0; i < EPT; i += 2) {
        float q0 = fminf(fmaxf(rintf(__fdiv_rn(xhv[i], scale)), -8.f), 7.f);
        float q1 = fminf(fmaxf(rintf(__fdiv_rn(xhv[i + 1], scale)), -8.f), 7.f);
        const uint32_t u0 = (uint32_t)((int)q0 + 8), u1 = (uint32_t)((int)q1 + 8);
        nib[i / 8] |= (u0 | (u1 << 4)) << ((i % 8) * 4);
        const __nv_fp8x2_storage_t f8 =
            __nv_cvt_float2_to_fp8x2(make_float2(q0, q1), __NV_SATFINITE, __NV_E4M3);
        if ((i % 4) == 0) e4[i / 4] = (uint32_t)f8;
        else e4[i / 4] |= (uint32_t)f8 << 16;
      }
      if (grow < p.M) {
        const int kc = k0 + qcol;
        if (p.packed) {
          uint8_t* dst = p.packed + (int64_t)grow * (p.K_pad / 2) + kc / 2;
          if constexpr (EPT == 8) *reinterpret_cast<uint32_t*>(dst) = nib[0];
          else *reinterpret_cast<uint2*>(dst) = make_uint2(nib[0], nib[1]);
        }
        if (p.codes) {
          uint8_t* dst = p.codes + (int64_t)grow * p.K_pad + kc;
          if constexpr (EPT == 8) *reinterpret_cast<uint2*>(dst) = make_uint2(e4[0], e4[1]);
          else *reinterpret_cast<uint4*>(dst) = make_uint4(e4[0], e4[1], e4[2], e4[3]);
        }
        if ((tid % 8) == 0) {
          if (p.scales) p.scales[(int64_t)grow * (p.K_pad / G) + c] = __float2bfloat16_rn(scale);
          if (p.scales_t) {
#pragma unroll
            for (int h = 0; h < G / 64; ++h)
              p.scales_t[(int64_t)(k0 / 64 + h) * p.ld_ast + grow] = scale;
          }
        }
      }
    }
    __syncthreads();  // x_hat tile complete

    // ---- low-rank down-projection on tensor cores ----
    if (n_tiles > 0) {
      const __nv_bfloat16* wst = ws + st * r_tot * LD;
      const __nv_bfloat16* xst = xs + st * kBM * LD;
#pragma unroll
      for (int kk = 0; kk < G / 16; ++kk) {
        // A fragments: rows (lane % 16), column block (lane / 16) * 8
        const int ar = lane % 16, ac = kk * 16 + (lane / 16) * 8;
        uint32_t a_hat[4], a_raw[4];
        ldmatrix_x4(smem_u32(xh + ar * LD + ac), a_hat[0], a_hat[1], a_hat[2], a_hat[3]);
        if (p.lora_rank > 0)
          ldmatrix_x4(smem_u32(xst + ar * LD + ac), a_raw[0], a_raw[1], a_raw[2], a_raw[3]);
#pragma unroll
        for (int j = 0; j < kMaxTilesPerWarp; ++j) {
          const int t = warp + 4 * j;
          if (t < n_tiles) {
            const int br = t * 8 + (lane % 8), bc = kk * 16 + ((lane / 8) % 2) * 8;
            uint32_t b0, b1;
            ldmatrix_x2(smem_u32(wst + br * LD + bc), b0, b1);
            if (t * 8 < p.rank) mma_bf16_16816(acc[j], a_hat, b0, b1);
            else mma_bf16_16816(acc[j], a_raw, b0, b1);
          }
        }
      }
    }
  }
  cp_async_wait<0>();

  // ---- mid as bf16 hi/lo pair ----
  if (p.mid_hl) {
    const int g = lane / 4, t4 = lane % 4;
#pragma unroll
    for (int j = 0; j < kMaxTilesPerWarp; ++j) {
      const int t = warp + 4 * j;
      if (t < n_tiles) {
        const int col = t * 8 + 2 * t4;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int row = m0 + g + 8 * h;
          float v0 = acc[j][2 * h], v1 = acc[j][2 * h + 1];
          if (col >= p.rank) {
            v0 *= p.lora_col_scale[col - p.rank];
            v1 *= p.lora_col_scale[col + 1 - p.rank];
          }
          const __nv_bfloat16 h0 = __float2bfloat16_rn(v0), h1 = __float2bfloat16_rn(v1);
          const __nv_bfloat16 l0 = __float2bfloat16_rn(v0 - __bfloat162float(h0));
          const __nv_bfloat16 l1 = __float2bfloat16_rn(v1 - __bfloat162float(h1));
          if (row < p.M) {
            __nv_bfloat16* dst = p.mid_hl + (int64_t)row * p.R2;
            __nv_bfloat162 hp, lp;
            hp.x = h0; hp.y = h1; lp.x = l0; lp.y = l1;
            *reinterpret_cast<__nv_bfloat162*>(dst + col) = hp;
            *reinterpret_cast<__nv_bfloat162*>(dst + r_tot + col) = lp;
          }
        }
      }
    }
    // zero the padding columns [2 r_tot, R2)
    const int pad = p.R2 - 2 * r_tot;
    for (int i = tid; i < kBM * pad; i += kThreads) {
      const int r = i / pad, cidx = 2 * r_tot + i % pad;
      if (m0 + r < p.M) p.mid_hl[(int64_t)(m0 + r) * p.R2 + cidx] = __float2bfloat16_rn(0.f);
    }
  }
}

}  // namespace
}  // namespace svdq

extern "C" int svdq_act_quant(const void* x, int64_t ldx, const void* smooth, const void* l2,
                              int rank, const void* lora_down, const float* lora_col_scale,
                              int lora_rank, int M, int K_in, int K_pad, int a_group,
                              void* out_packed, void* out_scales, void* out_codes,
                              float* out_scales_t, int ld_ast, void* out_mid_hl, int R2,
                              cudaStream_t stream) {
  using namespace svdq;
  SVDQ_REQUIRE(x && smooth, "svdq_act_quant: x and smooth are required");
  SVDQ_REQUIRE(M >= 0 && K_in > 0 && K_pad >= K_in, "svdq_act_quant: need 0 < K_in <= K_pad");
  SVDQ_REQUIRE(a_group == 64 || a_group == 128, "svdq_act_quant: a_group must be 64 or 128");
  SVDQ_REQUIRE(K_pad % a_group == 0, "svdq_act_quant: K_pad must be a multiple of a_group");
  SVDQ_REQUIRE(K_in % 8 == 0, "svdq_act_quant: K_in must be a multiple of 8 (pad smooth/l2 at load)");
  SVDQ_REQUIRE(ldx >= K_in && ldx % 8 == 0, "svdq_act_quant: ldx must be >= K_in and a multiple of 8");
  SVDQ_REQUIRE(rank >= 0 && lora_rank >= 0 && rank % 8 == 0 && lora_rank % 8 == 0,
               "svdq_act_quant: rank and lora_rank must be non-negative multiples of 8");
  SVDQ_REQUIRE(rank + lora_rank <= 256, "svdq_act_quant: rank + lora_rank must be <= 256");
  SVDQ_REQUIRE(rank == 0 || l2, "svdq_act_quant: l2 is NULL");
  SVDQ_REQUIRE(lora_rank == 0 || (lora_down && lora_col_scale),
               "svdq_act_quant: lora_down / lora_col_scale are NULL");
  const int r_tot = rank + lora_rank;
  SVDQ_REQUIRE(!out_mid_hl || (R2 >= 2 * r_tot && R2 % 8 == 0),
               "svdq_act_quant: R2 must be >= 2*(rank+lora_rank) and a multiple of 8");
  SVDQ_REQUIRE(!out_scales_t || (ld_ast >= M && ld_ast % 4 == 0),
               "svdq_act_quant: ld_ast must be >= M and a multiple of 4");
  SVDQ_REQUIRE((reinterpret_cast<uintptr_t>(x) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(smooth) & 15u) == 0 &&
                   (!l2 || (reinterpret_cast<uintptr_t>(l2) & 15u) == 0) &&
                   (!lora_down || (reinterpret_cast<uintptr_t>(lora_down) & 15u) == 0),
               "svdq_act_quant: x, smooth, l2, lora_down must be 16-byte aligned");
  SVDQ_REQUIRE((!out_codes || (reinterpret_cast<uintptr_t>(out_codes) & 15u) == 0) &&
                   (!out_packed || (reinterpret_cast<uintptr_t>(out_packed) & 7u) == 0),
               "svdq_act_quant: output code buffers are misaligned");
  if (M == 0) return SVDQ_OK;

  ActQuantParams p;
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.ldx = ldx;
  p.smooth = static_cast<const __nv_bfloat16*>(smooth);
  p.l2 = static_cast<const __nv_bfloat16*>(l2);
  p.lora = static_cast<const __nv_bfloat16*>(lora_down);
  p.lora_col_scale = lora_col_scale;
  p.rank = rank;
  p.lora_rank = lora_rank;
  p.M = M;
  p.K_in = K_in;
  p.K_pad = K_pad;
  p.packed = static_cast<uint8_t*>(out_packed);
  p.scales = static_cast<__nv_bfloat16*>(out_scales);
  p.codes = static_cast<uint8_t*>(out_codes);
  p.scales_t = out_scales_t;
  p.ld_ast = ld_ast;
  p.mid_hl = r_tot > 0 ? static_cast<__nv_bfloat16*>(out_mid_hl) : nullptr;
  p.R2 = R2;

  const int grid = (M + kBM - 1) / kBM;
  if (a_group == 64) {
    constexpr int LD = Smem<64>::LD;
    const size_t smem = sizeof(__nv_bfloat16) *
                        (size_t)(kStages * kBM * LD + kStages * r_tot * LD + kStages * 64 + kBM * LD);
    cudaFuncSetAttribute(act_quant_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    act_quant_kernel<64><<<grid, kThreads, smem, stream>>>(p);
  } else {
    constexpr int LD = Smem<128>::LD;
    const size_t smem = sizeof(__nv_bfloat16) *
                        (size_t)(kStages * kBM * LD + kStages * r_tot * LD + kStages * 128 + kBM * LD);
    cudaFuncSetAttribute(act_quant_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    act_quant_kernel<128><<<grid, kThreads, smem, stream>>>(p);
  }
  return check_launch("svdq_act_quant launch");
}
