// Load-time operand preparation for the linear GEMM.
//
// The checkpoint stores the residual weight as packed INT4 (q + 8 per nibble,
// even k in the low nibble; pack.py:47-56) with one scale per (row, group)
// (convert_simulated.py:201-204).  The GEMM consumes w16 = fp16(q * scale):
// q has at most 3 significant bits and a bf16 scale 8, so the product is exact
// in fp16 for bf16 scales (fp16 / fp32 scales round once, to nearest).
#include "svdq_common.cuh"

namespace svdq {
namespace {

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }

// Each thread expands 8 packed bytes (16 codes) of one row into 16 fp16 values.
template <typename T>
__global__ void repack_w16_kernel(const uint8_t* __restrict__ qw, const T* __restrict__ sc,
                                  __half* __restrict__ out, int N, int K_pad, int w_group) {
  const int64_t per_row = K_pad / 16;  // 16-code units per row
  const int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (u >= (int64_t)N * per_row) return;
  const int n = (int)(u / per_row);
  const int k0 = (int)(u % per_row) * 16;
  const float s = to_f32<T>(sc[(int64_t)n * (K_pad / w_group) + k0 / w_group]);  // w_group % 16 == 0
  const uint2 v = *reinterpret_cast<const uint2*>(qw + (int64_t)n * (K_pad / 2) + k0 / 2);
  uint32_t w[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t byte = ((j < 4 ? v.x : v.y) >> ((j % 4) * 8)) & 0xFF;
    const float q0 = (float)((int)(byte & 0xF) - 8), q1 = (float)((int)(byte >> 4) - 8);
    __half2 h = __floats2half2_rn(q0 * s, q1 * s);
    w[j] = *reinterpret_cast<uint32_t*>(&h);
  }
  uint4* o = reinterpret_cast<uint4*>(out + (int64_t)n * K_pad + k0);
  o[0] = make_uint4(w[0], w[1], w[2], w[3]);
  o[1] = make_uint4(w[4], w[5], w[6], w[7]);
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
                                  int K_pad, int w_group, void* out_w16, cudaStream_t stream) {
  using namespace svdq;
  SVDQ_REQUIRE(qweight && scales && out_w16, "svdq_repack_weight: null pointer");
  SVDQ_REQUIRE(N > 0 && K_pad > 0 && K_pad % 64 == 0, "svdq_repack_weight: K_pad must be a positive multiple of 64");
  SVDQ_REQUIRE(w_group > 0 && w_group % 16 == 0 && K_pad % w_group == 0,
               "svdq_repack_weight: w_group must be a multiple of 16 dividing K_pad");
  SVDQ_REQUIRE((reinterpret_cast<uintptr_t>(qweight) & 7u) == 0 &&
                   (reinterpret_cast<uintptr_t>(out_w16) & 15u) == 0,
               "svdq_repack_weight: qweight must be 8-byte and out_w16 16-byte aligned");
  const int64_t units = (int64_t)N * (K_pad / 16);
  const int threads = 256;
  const unsigned blocks = (unsigned)((units + threads - 1) / threads);
  __half* out = static_cast<__half*>(out_w16);
  const uint8_t* qw = static_cast<const uint8_t*>(qweight);
  switch (scale_dtype) {
    case SVDQ_BF16:
      repack_w16_kernel<<<blocks, threads, 0, stream>>>(qw, static_cast<const __nv_bfloat16*>(scales), out, N, K_pad, w_group);
      break;
    case SVDQ_FP16:
      repack_w16_kernel<<<blocks, threads, 0, stream>>>(qw, static_cast<const __half*>(scales), out, N, K_pad, w_group);
      break;
    case SVDQ_FP32:
      repack_w16_kernel<<<blocks, threads, 0, stream>>>(qw, static_cast<const float*>(scales), out, N, K_pad, w_group);
      break;
    default:
      return set_error(SVDQ_ERR_INVALID_ARGUMENT, "svdq_repack_weight: scale_dtype must be bf16, fp16 or fp32");
  }
  return check_launch("svdq_repack_weight");
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
