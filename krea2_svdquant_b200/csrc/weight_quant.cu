// Converter-side weight quantization on the GPU: the layer residual (fp32,
// [N, K]) -> packed INT4 codes [N, K_pad/2] + group scales [N, K_pad/G], the
// checkpoint format.  Same arithmetic as the reference's
// quantize_symmetric_int4 on fp32 input followed by pack_int4
// (src/krea2_svdquant/quant/pack.py:6-23, 47-56) as the converter calls them
// (scripts/convert_simulated.py:197-203):
//   zero-pad K to a multiple of G; amax = max |w| per group; scale =
//   max(amax, 1e-8f) / 7 (IEEE fp32 division); q = rint(w / scale) (IEEE fp32
//   division, ties to even) clamped to [-8, 7]; nibble q + 8, even k low.
// The scales are written as fp32, or rounded once to fp16 / bf16 (the
// converter stores `scales.to(torch.float16)`).  Off the per-call path: this
// runs once per layer at conversion time, so the divisions are the IEEE
// intrinsic rather than a faster reformulation.
#include <algorithm>
#include <type_traits>

#include "svdq_common.cuh"

namespace svdq {
namespace {

constexpr int kEPT = 8;  // elements per thread: one 32-byte fp32 read, one 4-byte packed write

template <int G, typename ScaleT>
__global__ void __launch_bounds__(256) quantize_weight_kernel(const float* __restrict__ w, int64_t ldw, int N, int K,
                                                              int K_pad, uint8_t* __restrict__ packed,
                                                              ScaleT* __restrict__ scales) {
  constexpr int TPG = G / kEPT;  // threads per group (8 or 16), aligned within a warp
  const int64_t per_row = K_pad / kEPT;
  const int64_t total = (int64_t)N * per_row;
  // every lane runs the same number of iterations so the group shuffles stay full-warp
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t iters = (total + stride - 1) / stride;
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  for (int64_t it = 0; it < iters; ++it, i += stride) {
    const bool live = i < total;
    const int64_t row = live ? i / per_row : 0;
    const int col = live ? (int)(i % per_row) * kEPT : 0;
    float v[kEPT];
#pragma unroll
    for (int e = 0; e < kEPT; ++e) v[e] = 0.f;
    if (live) {
      const float* src = w + row * ldw + col;
      if (col + kEPT <= K && (reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
        const float4 a = *reinterpret_cast<const float4*>(src);
        const float4 b = *reinterpret_cast<const float4*>(src + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      } else {
#pragma unroll
        for (int e = 0; e < kEPT; ++e)
          if (col + e < K) v[e] = src[e];
      }
    }
    float amax = 0.f;
#pragma unroll
    for (int e = 0; e < kEPT; ++e) amax = fmaxf(amax, fabsf(v[e]));
#pragma unroll
    for (int o = 1; o < TPG; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float scale = __fdiv_rn(fmaxf(amax, 1e-8f), 7.0f);
    uint32_t word = 0;
#pragma unroll
    for (int e = 0; e < kEPT; ++e) {
      const float q = fminf(fmaxf(rintf(__fdiv_rn(v[e], scale)), -8.f), 7.f);
      word |= (uint32_t)((int)q + 8) << (4 * e);
    }
    if (live) {
      *reinterpret_cast<uint32_t*>(packed + row * (K_pad / 2) + col / 2) = word;
      if (col % G == 0) {
        ScaleT* dst = scales + row * (K_pad / G) + col / G;
        if constexpr (std::is_same<ScaleT, float>::value) *dst = scale;
        else if constexpr (std::is_same<ScaleT, __half>::value) *dst = __float2half_rn(scale);
        else *dst = __float2bfloat16_rn(scale);
      }
    }
  }
}

template <int G>
int launch_g(const float* w, int64_t ldw, int N, int K, int K_pad, uint8_t* packed, void* scales, int dtype,
             cudaStream_t stream) {
  const int64_t total = (int64_t)N * (K_pad / kEPT);
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, (int64_t)num_sms() * 16);
  switch (dtype) {
    case SVDQ_FP32:
      quantize_weight_kernel<G, float><<<blocks, 256, 0, stream>>>(w, ldw, N, K, K_pad, packed,
                                                                     static_cast<float*>(scales));
      break;
    case SVDQ_FP16:
      quantize_weight_kernel<G, __half><<<blocks, 256, 0, stream>>>(w, ldw, N, K, K_pad, packed,
                                                                      static_cast<__half*>(scales));
      break;
    default:
      quantize_weight_kernel<G, __nv_bfloat16><<<blocks, 256, 0, stream>>>(w, ldw, N, K, K_pad, packed,
                                                                             static_cast<__nv_bfloat16*>(scales));
  }
  return check_launch("svdq_quantize_weight launch");
}

}  // namespace
}  // namespace svdq

extern "C" int svdq_quantize_weight(const float* w, int64_t ldw, int N, int K, int group, void* out_packed,
                                    void* out_scales, int scale_dtype, cudaStream_t stream) {
  using namespace svdq;
  SVDQ_REQUIRE(w && out_packed && out_scales, "svdq_quantize_weight: NULL pointer");
  SVDQ_REQUIRE(N >= 0 && K > 0 && ldw >= K, "svdq_quantize_weight: need K > 0 and ldw >= K");
  SVDQ_REQUIRE(group == 64 || group == 128, "svdq_quantize_weight: group must be 64 or 128");
  SVDQ_REQUIRE(scale_dtype == SVDQ_FP32 || scale_dtype == SVDQ_FP16 || scale_dtype == SVDQ_BF16,
               "svdq_quantize_weight: scale_dtype must be SVDQ_FP32, SVDQ_FP16 or SVDQ_BF16");
  SVDQ_REQUIRE((reinterpret_cast<uintptr_t>(out_packed) & 3u) == 0, "svdq_quantize_weight: packed must be 4-byte aligned");
  if (N == 0) return SVDQ_OK;
  const int K_pad = (K + group - 1) / group * group;
  auto* packed = static_cast<uint8_t*>(out_packed);
  return group == 64 ? launch_g<64>(w, ldw, N, K, K_pad, packed, out_scales, scale_dtype, stream)
                     : launch_g<128>(w, ldw, N, K, K_pad, packed, out_scales, scale_dtype, stream);
}
