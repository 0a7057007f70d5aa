// Activation pass of the SVDQuant linear (sm_100a).
//
// W4A4 mode: one pass over x [M, K_in] bf16 produces, per 32-row band and
// 128-column chunk:
//   x_hat = bf16(x / smooth)                             (svd.py:122)
//   q     = clamp(rint(x_hat / scale), -8, 7) per group  (pack.py:6-23)
//   scale = bf16(max(amax, bf16(1e-8)) / 7)              (pack.py:20)
//   packed nibbles (q + 8, even k low)                   (pack.py:47-56)
//   a16   = fp16(q * scale): the dequantized activation, exact in fp16
//   mid   = [x_hat @ l2^T | (x @ lora_down^T) * col_scale] (svd.py:159, linear.py:45)
//           written as a bf16 hi/lo pair so the GEMM's bf16 MMA keeps ~16 mantissa bits.
// W4A16 mode: a16 = fp16(fp32(x) / fp32(smooth)) (the reference run in fp32,
// svd.py:122 on float inputs) and mid from the fp16 x_hat against l2 converted
// to fp16 (exact for bf16 values in fp16 range).
// The down-projection runs on mma.sync tensor cores from shared memory; loads
// are a cp.async ring of 128-column chunks.
//
// W4A4 divisions must round exactly like float32 IEEE division followed by the
// reference's rounding (bf16 for x_hat, rint for q).  Each quotient is first
// formed as a product with the correctly rounded reciprocal; that product is
// within 2 ulp of the correctly rounded quotient, so the final rounding can
// only differ when the product lies within a few ulp of a rounding boundary
// (a bf16 midpoint, or a half-integer).  Those rare elements are recomputed
// with the IEEE division intrinsic __fdiv_rn.
#include <cuda_fp8.h>

#include "svdq_common.cuh"

namespace svdq {
namespace {

constexpr int kBM = 32;         // rows per CTA
constexpr int kThreads = 512;   // 16 warps
constexpr int kChunk = 128;     // columns per pipeline stage
constexpr int kLD = kChunk + 8; // padded smem row (bf16) so ldmatrix rows hit distinct banks
constexpr int kTilesPerWarp = 4;  // 8 column-tile sets x 4 tiles x 8 columns: r_tot <= 256

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
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

__device__ __forceinline__ void mma_f16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Near-boundary tests for the reciprocal-product quotients (see file comment).
// bf16 rounding of a float32 depends on its low 16 bits against 0x8000; a
// product within 2.5 ulp of the exact quotient can only round differently when
// its low bits are within 8 of 0x8000.
__device__ __forceinline__ bool near_bf16_midpoint(float t) {
  return ((__float_as_uint(t) & 0xFFFFu) - 0x7FF8u) < 0x10u;
}
// rint of a value below 8 in magnitude: the product is within 2.5 * 2^-21 of the
// exact quotient, so rint can only differ when it lies within 2^-19 of a half-integer.
__device__ __forceinline__ bool near_half_integer(float t, float r) {
  return 0.5f - fabsf(t - r) < 1.9073486e-06f;
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
  __half* a16;                 // [M, K_pad] fp16 GEMM operand
  __nv_bfloat16* mid_hl;       // [M, R2]
  int R2;
};

template <int G, int STAGES, bool W4A16>
__global__ void __launch_bounds__(kThreads) act_quant_kernel(const ActQuantParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int r_tot = p.rank + p.lora_rank;
  const int n_chunks = (p.K_pad + kChunk - 1) / kChunk;
  // layout: rsm[n_chunks * kChunk] fp32 (1/smooth), xs[STAGES][kBM][kLD], ws[STAGES][r_tot][kLD], xh[kBM][kLD]
  float* rsm = reinterpret_cast<float*>(smem_raw);
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(rsm + n_chunks * kChunk);
  __nv_bfloat16* ws = xs + STAGES * kBM * kLD;
  __nv_bfloat16* xh = ws + STAGES * r_tot * kLD;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int m0 = blockIdx.x * kBM;

  auto load_chunk = [&](int c) {
    const int st = c % STAGES;
    const int k0 = c * kChunk;
    constexpr int SEG = kChunk / 8;  // 16-byte segments per row
    for (int i = tid; i < kBM * SEG; i += kThreads) {
      const int r = i / SEG, s = i % SEG;
      const int col = k0 + s * 8, row = m0 + r;
      int bytes = 0;
      const __nv_bfloat16* src = p.x;
      if (row < p.M && col < p.K_in) {
        bytes = min(16, (p.K_in - col) * 2);
        src = p.x + (int64_t)row * p.ldx + col;
      }
      cp_async16(smem_u32(xs + (st * kBM + r) * kLD + s * 8), src, bytes);
    }
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
      cp_async16(smem_u32(ws + (st * r_tot + r) * kLD + s * 8), src, bytes);
    }
  };

#pragma unroll 1
  for (int c = 0; c < STAGES - 1; ++c) {
    if (c < n_chunks) load_chunk(c);
    cp_async_commit();
  }
  // correctly rounded reciprocals of the smoothing scale, once per CTA
  for (int k = tid; k < n_chunks * kChunk; k += kThreads)
    rsm[k] = k < p.K_in ? __frcp_rn(__bfloat162float(p.smooth[k])) : 0.f;

  // MMA work split: warp -> m-tile (warp & 1) and column tiles (warp >> 1) + 8 j
  const int mt = warp & 1;
  const int tset = warp >> 1;
  const int n_tiles = r_tot / 8;
  float acc[kTilesPerWarp][4];
#pragma unroll
  for (int j = 0; j < kTilesPerWarp; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;

  const float eps = __bfloat162float(__float2bfloat16_rn(1e-8f));
  const int qrow = tid / 16;        // quant step: 16 threads per row, 8 columns each
  const int cc = (tid % 16) * 8;    // column within the chunk
  const int grow = m0 + qrow;

#pragma unroll 1
  for (int c = 0; c < n_chunks; ++c) {
    const int st = c % STAGES;
    cp_async_wait<STAGES - 2>();
    __syncthreads();  // chunk c landed; everyone finished chunk c-1
    if (c + STAGES - 1 < n_chunks) load_chunk(c + STAGES - 1);
    cp_async_commit();

    const int col0 = c * kChunk + cc;
    if constexpr (W4A16) {
      // ---- x_hat = fp16(fp32 division), and l2 rows of this chunk to fp16 ----
      const uint4 xv = *reinterpret_cast<const uint4*>(xs + (st * kBM + qrow) * kLD + cc);
      const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&xv);
      uint32_t hw[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(x2[i]);
        const int col = col0 + 2 * i;
        const float v0 = col < p.K_in ? __fdiv_rn(f.x, __bfloat162float(p.smooth[col])) : 0.f;
        const float v1 = col + 1 < p.K_in ? __fdiv_rn(f.y, __bfloat162float(p.smooth[col + 1])) : 0.f;
        __half2 h = __floats2half2_rn(v0, v1);
        hw[i] = *reinterpret_cast<uint32_t*>(&h);
      }
      const uint4 hv = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      *reinterpret_cast<uint4*>(xh + qrow * kLD + cc) = hv;
      if (col0 < p.K_pad && grow < p.M && p.a16)
        *reinterpret_cast<uint4*>(p.a16 + (int64_t)grow * p.K_pad + col0) = hv;
      // the l2 rows are consumed by an fp16 MMA in this mode
      for (int i = tid; i < p.rank * (kChunk / 8); i += kThreads) {
        const int r = i / (kChunk / 8), sg = i % (kChunk / 8);
        uint4* ptr = reinterpret_cast<uint4*>(ws + (st * r_tot + r) * kLD + sg * 8);
        uint4 v = *ptr;
        uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&w[e]));
          __half2 h = __floats2half2_rn(f.x, f.y);
          w[e] = *reinterpret_cast<uint32_t*>(&h);
        }
        *ptr = v;
      }
    } else {
    // ---- smoothing + group quantization (bit-exact with the reference) ----
      {
        const uint4 xv = *reinterpret_cast<const uint4*>(xs + (st * kBM + qrow) * kLD + cc);
        const float4 r0 = *reinterpret_cast<const float4*>(rsm + col0);
        const float4 r1 = *reinterpret_cast<const float4*>(rsm + col0 + 4);
        const float rv[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
        const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&xv);
        float xf[8], t[8];
        bool slow = false;
  #pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __bfloat1622float2(x2[i]);
          xf[2 * i] = f.x;
          xf[2 * i + 1] = f.y;
        }
  #pragma unroll
        for (int i = 0; i < 8; ++i) {
          t[i] = xf[i] * rv[i];
          slow |= near_bf16_midpoint(t[i]);
        }
        if (slow) {
  #pragma unroll
          for (int i = 0; i < 8; ++i)
            if (near_bf16_midpoint(t[i]) && col0 + i < p.K_in)
              t[i] = __fdiv_rn(xf[i], __bfloat162float(p.smooth[col0 + i]));
        }
        uint32_t hw[4];
        float xhv[8];
        float amax = 0.f;
  #pragma unroll
        for (int i = 0; i < 4; ++i) {
          __nv_bfloat162 pr = __floats2bfloat162_rn(t[2 * i], t[2 * i + 1]);
          hw[i] = *reinterpret_cast<uint32_t*>(&pr);
          const float2 f = __bfloat1622float2(pr);
          xhv[2 * i] = f.x;
          xhv[2 * i + 1] = f.y;
          amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
        }
        *reinterpret_cast<uint4*>(xh + qrow * kLD + cc) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
  #pragma unroll
        for (int o = 1; o < G / 8; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float scale = __bfloat162float(__float2bfloat16_rn(__fdiv_rn(fmaxf(amax, eps), 7.0f)));
        const float rs = __frcp_rn(scale);
        // rint and the offset-binary code in one add: for |t| < 2^22, t + 1.5*2^23 + 8
        // rounds t to the nearest integer (ties to even) and its low mantissa bits
        // hold rint(t) + 8.  |x_hat / scale| <= 7 * (1 + 2^-8), so rint(t) is in
        // [-7, 7] and the reference's clamp to [-8, 7] never binds.
        constexpr float kMagic = 12582920.0f;  // 1.5 * 2^23 + 8
        float tq[8], qv[8];
        uint32_t u[8];
        slow = false;
  #pragma unroll
        for (int i = 0; i < 8; ++i) {
          tq[i] = xhv[i] * rs;
          const float m = tq[i] + kMagic;
          qv[i] = m - kMagic;  // rint(tq), exact
          u[i] = __float_as_uint(m);
          slow |= near_half_integer(tq[i], qv[i]);
        }
        if (slow) {
  #pragma unroll
          for (int i = 0; i < 8; ++i) {
            if (near_half_integer(tq[i], qv[i])) {
              const float m = __fdiv_rn(xhv[i], scale) + kMagic;
              qv[i] = m - kMagic;
              u[i] = __float_as_uint(m);
            }
          }
        }
        uint32_t nib = 0, aw[4];
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          nib |= ((u[i] & 0xFu) | ((u[i + 1] & 0xFu) << 4)) << (i * 4);
          // q * scale is exact in fp32 and in fp16 (at most 11 significant bits)
          __half2 h = __floats2half2_rn(qv[i] * scale, qv[i + 1] * scale);
          aw[i / 2] = *reinterpret_cast<uint32_t*>(&h);
        }
        if (col0 < p.K_pad && grow < p.M) {
          if (p.packed) *reinterpret_cast<uint32_t*>(p.packed + (int64_t)grow * (p.K_pad / 2) + col0 / 2) = nib;
          if (p.a16)
            *reinterpret_cast<uint4*>(p.a16 + (int64_t)grow * p.K_pad + col0) = make_uint4(aw[0], aw[1], aw[2], aw[3]);
          if ((tid % (G / 8)) == 0 && p.scales)
            p.scales[(int64_t)grow * (p.K_pad / G) + col0 / G] = __float2bfloat16_rn(scale);
        }
      }
    }
    __syncthreads();  // x_hat tile complete

    // ---- low-rank down-projection on tensor cores ----
    if (tset < n_tiles) {
      const __nv_bfloat16* wst = ws + st * r_tot * kLD;
      const __nv_bfloat16* xst = xs + (st * kBM + mt * 16) * kLD;
      const __nv_bfloat16* xht = xh + (mt * 16) * kLD;
#pragma unroll 2
      for (int kk = 0; kk < kChunk / 16; ++kk) {
        const int ar = lane % 16, ac = kk * 16 + (lane / 16) * 8;
        uint32_t a_hat[4], a_raw[4];
        ldmatrix_x4(smem_u32(xht + ar * kLD + ac), a_hat);
        if (p.lora_rank > 0) ldmatrix_x4(smem_u32(xst + ar * kLD + ac), a_raw);
#pragma unroll
        for (int j = 0; j < kTilesPerWarp; ++j) {
          const int t = tset + 8 * j;
          if (t < n_tiles) {
            const int br = t * 8 + (lane % 8), bc = kk * 16 + ((lane / 8) % 2) * 8;
            uint32_t b0, b1;
            ldmatrix_x2(smem_u32(wst + br * kLD + bc), b0, b1);
            if (t * 8 < p.rank) {
              if constexpr (W4A16) mma_f16_16816(acc[j], a_hat, b0, b1);
              else mma_bf16_16816(acc[j], a_hat, b0, b1);
            } else {
              mma_bf16_16816(acc[j], a_raw, b0, b1);
            }
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
    for (int j = 0; j < kTilesPerWarp; ++j) {
      const int t = tset + 8 * j;
      if (t < n_tiles) {
        const int col = t * 8 + 2 * t4;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int row = m0 + mt * 16 + g + 8 * h;
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
    const int pad = p.R2 - 2 * r_tot;
    for (int i = tid; i < kBM * pad; i += kThreads) {
      const int r = i / pad, cidx = 2 * r_tot + i % pad;
      if (m0 + r < p.M) p.mid_hl[(int64_t)(m0 + r) * p.R2 + cidx] = __float2bfloat16_rn(0.f);
    }
  }
}

constexpr size_t kSmemBudget = 220 * 1024;

size_t smem_bytes(int stages, int r_tot, int k_pad) {
  const size_t n_chunks = (size_t)((k_pad + kChunk - 1) / kChunk);
  return sizeof(float) * n_chunks * kChunk +
         sizeof(__nv_bfloat16) * (size_t)(stages * kBM * kLD + stages * r_tot * kLD + kBM * kLD);
}

template <int G, int STAGES, bool W4A16>
int launch(const ActQuantParams& prm, int r_tot, cudaStream_t stream) {
  const size_t smem = smem_bytes(STAGES, r_tot, prm.K_pad);
  auto kern = act_quant_kernel<G, STAGES, W4A16>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return check_cuda(e, "svdq_act_quant: shared memory attribute");
  const int grid = (prm.M + kBM - 1) / kBM;
  kern<<<grid, kThreads, smem, stream>>>(prm);
  return check_launch("svdq_act_quant launch");
}

template <int G, bool W4A16>
int launch_g(const ActQuantParams& prm, int r_tot, cudaStream_t stream) {
  // deepest ring that fits in the shared-memory budget
  if (smem_bytes(4, r_tot, prm.K_pad) <= kSmemBudget) return launch<G, 4, W4A16>(prm, r_tot, stream);
  if (smem_bytes(3, r_tot, prm.K_pad) <= kSmemBudget) return launch<G, 3, W4A16>(prm, r_tot, stream);
  if (smem_bytes(2, r_tot, prm.K_pad) <= kSmemBudget) return launch<G, 2, W4A16>(prm, r_tot, stream);
  return set_error(SVDQ_ERR_UNSUPPORTED, "svdq_act_quant: K_pad / rank too large for shared memory");
}

}  // namespace
}  // namespace svdq

namespace svdq {
namespace {

int validate_common(const void* x, int64_t ldx, const void* smooth, const void* l2, int rank, const void* lora_down,
                    const float* lora_col_scale, int lora_rank, int M, int K_in, int K_pad, void* out_a16,
                    void* out_mid_hl, int R2, const char* who) {
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
  if (out_a16 && ((reinterpret_cast<uintptr_t>(out_a16) & 15u) || K_pad % 8 != 0))
    return bad("a16 must be 16-byte aligned with K_pad a multiple of 8");
  return SVDQ_OK;
}

ActQuantParams make_params(const void* x, int64_t ldx, const void* smooth, const void* l2, int rank,
                           const void* lora_down, const float* lora_col_scale, int lora_rank, int M, int K_in,
                           int K_pad, void* out_packed, void* out_scales, void* out_a16, void* out_mid_hl, int R2) {
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
  p.a16 = static_cast<__half*>(out_a16);
  p.mid_hl = (rank + lora_rank) > 0 ? static_cast<__nv_bfloat16*>(out_mid_hl) : nullptr;
  p.R2 = R2;
  return p;
}

}  // namespace
}  // namespace svdq

extern "C" int svdq_act_quant(const void* x, int64_t ldx, const void* smooth, const void* l2, int rank,
                              const void* lora_down, const float* lora_col_scale, int lora_rank, int M, int K_in,
                              int K_pad, int a_group, void* out_packed, void* out_scales, void* out_a16,
                              void* out_mid_hl, int R2, cudaStream_t stream) {
  using namespace svdq;
  int st = validate_common(x, ldx, smooth, l2, rank, lora_down, lora_col_scale, lora_rank, M, K_in, K_pad, out_a16,
                           out_mid_hl, R2, "svdq_act_quant");
  if (st) return st;
  SVDQ_REQUIRE(a_group == 64 || a_group == 128, "svdq_act_quant: a_group must be 64 or 128");
  SVDQ_REQUIRE(K_pad % a_group == 0, "svdq_act_quant: K_pad must be a multiple of a_group");
  SVDQ_REQUIRE(!out_packed || (reinterpret_cast<uintptr_t>(out_packed) & 3u) == 0,
               "svdq_act_quant: packed output must be 4-byte aligned");
  if (M == 0) return SVDQ_OK;
  const ActQuantParams p = make_params(x, ldx, smooth, l2, rank, lora_down, lora_col_scale, lora_rank, M, K_in,
                                       K_pad, out_packed, out_scales, out_a16, out_mid_hl, R2);
  const int r_tot = rank + lora_rank;
  return a_group == 64 ? launch_g<64, false>(p, r_tot, stream) : launch_g<128, false>(p, r_tot, stream);
}

extern "C" int svdq_w4a16_prep(const void* x, int64_t ldx, const void* smooth, const void* l2, int rank,
                               const void* lora_down, const float* lora_col_scale, int lora_rank, int M, int K_in,
                               int K_pad, void* out_a16, void* out_mid_hl, int R2, cudaStream_t stream) {
  using namespace svdq;
  int st = validate_common(x, ldx, smooth, l2, rank, lora_down, lora_col_scale, lora_rank, M, K_in, K_pad, out_a16,
                           out_mid_hl, R2, "svdq_w4a16_prep");
  if (st) return st;
  SVDQ_REQUIRE(out_a16, "svdq_w4a16_prep: out_a16 is required");
  SVDQ_REQUIRE(K_pad % 64 == 0, "svdq_w4a16_prep: K_pad must be a multiple of 64");
  if (M == 0) return SVDQ_OK;
  const ActQuantParams p = make_params(x, ldx, smooth, l2, rank, lora_down, lora_col_scale, lora_rank, M, K_in,
                                       K_pad, nullptr, nullptr, out_a16, out_mid_hl, R2);
  return launch_g<64, true>(p, rank + lora_rank, stream);
}
