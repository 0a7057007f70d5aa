// Load-time operand preparation for the W4A4 GEMM.
//
// The checkpoint stores the residual weight as packed INT4 (q + 8 per nibble,
// even k in the low nibble; pack.py:47-56) with one scale per (row, group)
// (convert_simulated.py:201-204).  The GEMM consumes the same integers as e4m3
// bytes (every integer in [-8, 7] is exact in e4m3) and the scales transposed
// to [K_pad/64, N] fp32, one row per 64-wide K group, so a 128x256 output tile
// reads its scales as contiguous TMA boxes.
#include <cuda_fp8.h>

#include "svdq_common.cuh"

namespace svdq {
namespace {

// e4m3 bytes of q = u - 8 for every nibble value u (offset-binary code).
__device__ __forceinline__ uint32_t nib_to_e4m3_pair(uint32_t byte) {
  const float q0 = (float)((int)(byte & 0xF) - 8);
  const float q1 = (float)((int)(byte >> 4) - 8);
  return (uint32_t)__nv_cvt_float2_to_fp8x2(make_float2(q0, q1), __NV_SATFINITE, __NV_E4M3);
}

// Each thread expands 8 packed bytes (16 codes).
__global__ void repack_codes_kernel(const uint8_t* __restrict__ qw, uint8_t* __restrict__ out,
                                    int64_t n_bytes) {
  const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (i >= n_bytes) return;
  if (i + 8 <= n_bytes) {
    const uint2 v = *reinterpret_cast<const uint2*>(qw + i);
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t word = j < 2 ? v.x : v.y;
      const uint32_t b0 = (word >> ((j % 2) * 16)) & 0xFF;
      const uint32_t b1 = (word >> ((j % 2) * 16 + 8)) & 0xFF;
      w[j] = nib_to_e4m3_pair(b0) | (nib_to_e4m3_pair(b1) << 16);
    }
    *reinterpret_cast<uint4*>(out + 2 * i) = make_uint4(w[0], w[1], w[2], w[3]);
  } else {
    for (int64_t k = i; k < n_bytes; ++k) {
      const uint32_t pr = nib_to_e4m3_pair(qw[k]);
      out[2 * k] = (uint8_t)(pr & 0xFF);
      out[2 * k + 1] = (uint8_t)(pr >> 8);
    }
  }
}

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }

// out[g64][n] = scales[n][g64 * 64 / w_group]
template <typename T>
__global__ void repack_scales_kernel(const T* __restrict__ sc, float* __restrict__ out, int N,
                                     int n_g64, int n_gw, int ratio) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  const int g = blockIdx.y;
  if (n >= N || g >= n_g64) return;
  out[(int64_t)g * N + n] = to_f32<T>(sc[(int64_t)n * n_gw + g / ratio]);
}

// up_hl[n] = [l1[n] | lora_up[n] | l1[n] | lora_up[n] | 0 ...]
__global__ void build_up_hl_kernel(const __nv_bfloat16* __restrict__ l1, int rank,
                                   const __nv_bfloat16* __restrict__ lu, int lora_rank, int N,
                                   __nv_bfloat16* __restrict__ out, int R2) {
  const int n = blockIdx.y;
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N || j >= R2) return;
  const int r_tot = rank + lora_rank;
  __nv_bfloat16 v = __float2bfloat16_rn(0.f);
  if (j < 2 * r_tot) {
    const int c = j % r_tot;
    v = c < rank ? l1[(int64_t)n * rank + c] : lu[(int64_t)n * lora_rank + (c - rank)];
  }
  out[(int64_t)n * R2 + j] = v;
}

}  // namespace
}  // namespace svdq

extern "C" int svdq_repack_weight(const void* qweight, const void* scales, int scale_dtype, int N,
                                  int K_pad, int w_group, void* out_codes, float* out_scales_t,
                                  cudaStream_t stream) {
  using namespace svdq;
  SVDQ_REQUIRE(qweight && scales && out_codes && out_scales_t, "svdq_repack_weight: null pointer");
  SVDQ_REQUIRE(N > 0 && K_pad > 0 && K_pad % 64 == 0, "svdq_repack_weight: K_pad must be a positive multiple of 64");
  SVDQ_REQUIRE(w_group > 0 && w_group % 64 == 0 && K_pad % w_group == 0,
               "svdq_repack_weight: w_group must be a multiple of 64 dividing K_pad");
  SVDQ_REQUIRE((reinterpret_cast<uintptr_t>(qweight) & 7u) == 0 &&
                   (reinterpret_cast<uintptr_t>(out_codes) & 15u) == 0,
               "svdq_repack_weight: qweight must be 8-byte and out_codes 16-byte aligned");
  SVDQ_REQUIRE(N <= 65535, "svdq_repack_weight: N must be <= 65535");
  const int64_t n_bytes = (int64_t)N * (K_pad / 2);
  const int threads = 256;
  const int64_t blocks = ((n_bytes + 7) / 8 + threads - 1) / threads;
  repack_codes_kernel<<<(unsigned)blocks, threads, 0, stream>>>(
      static_cast<const uint8_t*>(qweight), static_cast<uint8_t*>(out_codes), n_bytes);
  int st = check_launch("svdq_repack_weight codes");
  if (st) return st;
  const int n_g64 = K_pad / 64, n_gw = K_pad / w_group, ratio = w_group / 64;
  dim3 grid((N + 255) / 256, n_g64);
  switch (scale_dtype) {
    case SVDQ_BF16:
      repack_scales_kernel<<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(scales),
                                                     out_scales_t, N, n_g64, n_gw, ratio);
      break;
    case SVDQ_FP16:
      repack_scales_kernel<<<grid, 256, 0, stream>>>(static_cast<const __half*>(scales),
                                                     out_scales_t, N, n_g64, n_gw, ratio);
      break;
    case SVDQ_FP32:
      repack_scales_kernel<<<grid, 256, 0, stream>>>(static_cast<const float*>(scales),
                                                     out_scales_t, N, n_g64, n_gw, ratio);
      break;
    default:
      return set_error(SVDQ_ERR_INVALID_ARGUMENT, "svdq_repack_weight: scale_dtype must be bf16, fp16 or fp32");
  }
  return check_launch("svdq_repack_weight scales");
}

extern "C" int svdq_build_up_hl(const void* l1, int rank, const void* lora_up, int lora_rank, int N,
                                void* out_up_hl, int R2, cudaStream_t stream) {
  using namespace svdq;
  SVDQ_REQUIRE(out_up_hl && N > 0, "svdq_build_up_hl: null output or N <= 0");
  SVDQ_REQUIRE(rank >= 0 && lora_rank >= 0, "svdq_build_up_hl: negative rank");
  SVDQ_REQUIRE(rank == 0 || l1, "svdq_build_up_hl: l1 is NULL");
  SVDQ_REQUIRE(lora_rank == 0 || lora_up, "svdq_build_up_hl: lora_up is NULL");
  SVDQ_REQUIRE(R2 >= 2 * (rank + lora_rank), "svdq_build_up_hl: R2 too small");
  SVDQ_REQUIRE(N <= 65535, "svdq_build_up_hl: N must be <= 65535");
  if (R2 == 0) return SVDQ_OK;
  dim3 grid((R2 + 127) / 128, N);
  build_up_hl_kernel<<<grid, 128, 0, stream>>>(static_cast<const __nv_bfloat16*>(l1), rank,
                                               static_cast<const __nv_bfloat16*>(lora_up), lora_rank,
                                               N, static_cast<__nv_bfloat16*>(out_up_hl), R2);
  return check_launch("svdq_build_up_hl");
}
