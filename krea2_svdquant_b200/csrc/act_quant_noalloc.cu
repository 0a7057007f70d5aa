// svdq_act_quant_noalloc: the W4A4 activation pass with its K-slice scratch in
// a file-scope device array instead of a caller-provided workspace.
//
// For callers that cannot allocate device memory at the call site: a C / FFI
// host that binds only this ABI inside a process whose device memory belongs
// to another framework, or a serving loop that forbids allocation after
// warm-up so that no request can block on a synchronizing allocation or fail
// on fragmentation.  The call allocates nothing: no cudaMalloc / cudaFree and
// no other allocating routine.  The scratch address is looked up with
// cudaGetSymbolAddress on the first call in each CUDA context (the device's
// primary context, or any other context the host made current), whatever
// that call's shape; when that first call would otherwise fall inside a
// stream capture, make one call of any shape before capturing.  The scratch
// holds kNoAllocScratchBytes; a call that needs more is rejected with
// SVDQ_ERR_UNSUPPORTED and names the size it needs.
// The scratch holds the K-slice partial sums, which need no clearing: every K
// slice writes all of its partials before the call's second launch reads them,
// and each call leaves its own partials behind.  All calls on one device
// share the one scratch array, so calls that overlap in time (on different
// streams, or from different host threads) race on it and must be serialized
// by the caller.
#include "svdq_common.cuh"

extern "C" size_t svdq_act_quant_workspace_bytes(int M, int K_pad, int rank, int lora_rank);
extern "C" int svdq_act_quant(const void* x, int64_t ldx, const void* smooth, const void* l2, int rank,
                              const void* lora_down, const float* lora_col_scale, int lora_rank, int M, int K_in,
                              int K_pad, int a_group, void* out_packed, void* out_scales, void* out_a16,
                              void* out_mid_hl, int R2, void* workspace, size_t workspace_bytes,
                              cudaStream_t stream);

namespace svdq {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB per device
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

// Device address of the scratch array in the current context.  The first call in a context looks
// it up with cudaGetSymbolAddress (with that context's device current); later calls reuse it.
int noalloc_scratch(void** out) {
  return symbol_address(reinterpret_cast<const void*>(&g_noalloc_scratch), out,
                        "svdq_act_quant_noalloc: scratch address");
}

}  // namespace
}  // namespace svdq

extern "C" size_t svdq_act_quant_noalloc_scratch_bytes(void) { return svdq::kNoAllocScratchBytes; }

extern "C" int svdq_act_quant_noalloc(const void* x, int64_t ldx, const void* smooth, const void* l2, int rank,
                                      const void* lora_down, const float* lora_col_scale, int lora_rank, int M,
                                      int K_in, int K_pad, int a_group, void* out_packed, void* out_scales,
                                      void* out_a16, void* out_mid_hl, int R2, cudaStream_t stream) {
  using namespace svdq;
  const size_t need = (out_mid_hl && rank + lora_rank > 0 && M > 0 && K_pad > 0 && rank >= 0 && lora_rank >= 0)
                          ? svdq_act_quant_workspace_bytes(M, K_pad, rank, lora_rank)
                          : 0;
  if (need > kNoAllocScratchBytes)
    return set_error(SVDQ_ERR_UNSUPPORTED, "svdq_act_quant_noalloc: this call needs " + std::to_string(need) +
                                               " bytes of scratch but the static scratch holds " +
                                               std::to_string(kNoAllocScratchBytes) +
                                               " bytes; use svdq_act_quant with a caller-provided workspace");
  // looked up on every call, whether or not this call uses the scratch, so the one-time set-up of a
  // context happens on its first call of any shape
  void* scratch = nullptr;
  const int st = noalloc_scratch(&scratch);
  if (st) return st;
  return svdq_act_quant(x, ldx, smooth, l2, rank, lora_down, lora_col_scale, lora_rank, M, K_in, K_pad, a_group,
                        out_packed, out_scales, out_a16, out_mid_hl, R2, need > 0 ? scratch : nullptr, need, stream);
}
