// Host runtime pieces shared by all entry points: error strings, the device
// error word, tensor-map encoding through the driver entry point, SM count.
#include <atomic>
#include <cudaTypedefs.h>

#include <mutex>
#include <string>

#include "svdq_common.cuh"

namespace svdq {

static __device__ int g_device_error = 0;

namespace {
using PFN_ctx_get = CUresult (*)(CUcontext*);
PFN_ctx_get g_ctx_get = nullptr;
std::once_flag g_ctx_once;

// Symbol addresses cached per CUDA context: a device's primary context and any other context an
// FFI host makes current hold separate module instances, so the address of one is not valid in another.
struct CtxAddr {
  CUcontext ctx;
  const void* symbol;
  void* addr;
};
constexpr int kMaxCtxAddrs = 256;
CtxAddr g_ctx_addrs[kMaxCtxAddrs];
int g_ctx_addr_count = 0;
std::mutex g_ctx_addr_mutex;
}  // namespace

int current_context(CUcontext* out) {
  std::call_once(g_ctx_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_ctx_get = reinterpret_cast<PFN_ctx_get>(fn);
  });
  if (!g_ctx_get) return set_error(SVDQ_ERR_CUDA, "cuCtxGetCurrent entry point not found");
  CUcontext c = nullptr;
  if (g_ctx_get(&c) != CUDA_SUCCESS) return set_error(SVDQ_ERR_CUDA, "cuCtxGetCurrent failed");
  if (!c) {
    // nothing current yet on this thread: cudaSetDevice makes the device's primary context current
    int dev = 0;
    int st = check_cuda(cudaGetDevice(&dev), "current device");
    if (!st) st = check_cuda(cudaSetDevice(dev), "binding the current device's primary context");
    if (st) return st;
    if (g_ctx_get(&c) != CUDA_SUCCESS || !c) return set_error(SVDQ_ERR_CUDA, "no current CUDA context");
  }
  *out = c;
  return SVDQ_OK;
}

int symbol_address(const void* symbol, void** out, const char* what) {
  CUcontext ctx = nullptr;
  int st = current_context(&ctx);
  if (st) return st;
  std::lock_guard<std::mutex> lock(g_ctx_addr_mutex);
  for (int i = 0; i < g_ctx_addr_count; ++i)
    if (g_ctx_addrs[i].ctx == ctx && g_ctx_addrs[i].symbol == symbol) {
      *out = g_ctx_addrs[i].addr;
      return SVDQ_OK;
    }
  void* p = nullptr;
  st = check_cuda(cudaGetSymbolAddress(&p, symbol), what);
  if (st) return st;
  if (g_ctx_addr_count < kMaxCtxAddrs) g_ctx_addrs[g_ctx_addr_count++] = CtxAddr{ctx, symbol, p};
  *out = p;
  return SVDQ_OK;
}

int* device_error_word() {
  void* p = nullptr;
  if (symbol_address(reinterpret_cast<const void*>(&g_device_error), &p, "device error word address")) return nullptr;
  return static_cast<int*>(p);
}

static thread_local std::string t_last_error;

int set_error(int status, const std::string& msg) {
  t_last_error = msg;
  return status;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return SVDQ_OK;
  return set_error(SVDQ_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int check_launch(const char* what) { return check_cuda(cudaGetLastError(), what); }

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

int make_tma_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner,
                uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) return set_error(SVDQ_ERR_CUDA, "cuTensorMapEncodeTiled entry point not found");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    return set_error(SVDQ_ERR_INVALID_ARGUMENT, "TMA base address is not 16-byte aligned");
  if (row_stride_bytes % 16 != 0)
    return set_error(SVDQ_ERR_INVALID_ARGUMENT, "TMA row stride is not a multiple of 16 bytes");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(SVDQ_ERR_CUDA, "cuTensorMapEncodeTiled failed with code " + std::to_string((int)r));
  return SVDQ_OK;
}

int num_sms() {
  static std::atomic<int> cache[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  int c = cache[dev].load(std::memory_order_relaxed);
  if (c == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    c = n > 0 ? n : 148;
    cache[dev].store(c, std::memory_order_relaxed);
  }
  return c;
}

}  // namespace svdq

extern "C" {

const char* svdq_last_error(void) { return svdq::t_last_error.c_str(); }

const char* svdq_version(void) { return "svdq_b200 0.1"; }

int svdq_device_error(int* code, int clear) {
  if (!code) return svdq::set_error(SVDQ_ERR_INVALID_ARGUMENT, "code is NULL");
  int st = svdq::check_cuda(cudaDeviceSynchronize(), "svdq_device_error: synchronize");
  if (st) return st;
  st = svdq::check_cuda(cudaMemcpyFromSymbol(code, svdq::g_device_error, sizeof(int)),
                        "svdq_device_error: read");
  if (st) return st;
  if (clear) {
    int zero = 0;
    st = svdq::check_cuda(cudaMemcpyToSymbol(svdq::g_device_error, &zero, sizeof(int)),
                          "svdq_device_error: clear");
  }
  return st;
}

}  // extern "C"

namespace svdq {
namespace {

constexpr int kErrSelftestWait = 0x7E01;

// One CTA waits on an mbarrier that nothing arrives on, through the same bounded
// wait every kernel of this library uses, with a short limit.  The wait gives up,
// records kErrSelftestWait and the kernel exits normally.
__global__ void selftest_bounded_wait_kernel(unsigned long long limit_ns, int* err) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(smem_u32(&bar), 0, &abort_flag, err, kErrSelftestWait, limit_ns);
  __syncthreads();
}

}  // namespace
}  // namespace svdq

extern "C" int svdq_selftest_bounded_wait(int limit_us, cudaStream_t stream) {
  using namespace svdq;
  SVDQ_REQUIRE(limit_us >= 1 && limit_us <= 5000000, "svdq_selftest_bounded_wait: limit_us must be in [1, 5e6]");
  int* err = device_error_word();
  if (!err) return set_error(SVDQ_ERR_CUDA, "svdq_selftest_bounded_wait: device error word unavailable");
  selftest_bounded_wait_kernel<<<1, 32, 0, stream>>>((unsigned long long)limit_us * 1000ull, err);
  return check_launch("svdq_selftest_bounded_wait launch");
}
