// SVDQuant linear GEMM for sm_100a (tcgen05 + TMA + TMEM, CTA pairs).
//
//   out[m, n] = sum_k A[m,k] W[n,k] + sum_j mid_hl[m,j] up_hl[n,j] + bias[n]
//
// A and W are fp16 operands that hold the dequantized INT4 values exactly:
// A = fp16(q_a * s_a) from the activation pass (W4A4) or fp16(x / smooth)
// (W4A16), W = fp16(q_w * s_w) from the load-time weight preparation.  The
// product of a code in [-8, 7] (at most 3 significant bits) and a bf16 scale
// (8 significant bits) has at most 11 significant bits, so it is exact in
// fp16 whenever it lies in fp16's range; the MMA then sums exact products in
// fp32, which is the staged W4A4 result of the reference's README formula.
// Accumulating the whole K in TMEM keeps the tensor core's accumulator private:
// nothing reads TMEM between K steps (reading per-group partials out of TMEM
// while MMAs run is limited to a small fraction of TMEM bandwidth on B200).
//
// Persistent kernel launched as clusters of two CTAs.  A pair owns one 256x256
// output tile at a time; the even CTA issues cta_group::2 MMAs (M=256, N=256)
// whose A rows (128 per CTA) and W rows (128 per CTA) are split between the two
// CTAs' shared memory, so each operand byte crosses L2 once per pair.  Each
// CTA's TMEM receives its 128 rows x 256 columns; two accumulators let the
// epilogue of one tile overlap the MMAs of the next.  12 warps per CTA:
//   warp 0      TMA producer (both CTAs): per stage one 128-byte K slice (64
//               fp16) of the CTA's A rows and W half, counted on the even CTA's
//               barrier; then the low-rank stages (mid_hl x up_hl, bf16).
//   warp 1      TMEM allocator (both CTAs) and, in the even CTA, MMA issuer
//               (kind::f16: fp16 for the residual, bf16 for the low-rank term).
//   warps 4-11  epilogue (both CTAs): two warpgroups, 128 columns each; TMEM ->
//               registers -> + bias -> [op with an operand z: z + y, z * sigmoid(y),
//               silu(z) * y] -> bf16/fp32 -> global.
// Every mbarrier wait is bounded; a wait that runs out sets a CTA abort flag and
// the library's device error word, and all roles leave their loops, so both
// CTAs always reach the closing cluster barrier.
//
// Split tail.  Whole tiles fill as many complete waves over the pairs as they
// can; when the remaining tiles would leave most pairs idle for a last wave,
// their K iterations (residual stages, then low-rank stages) are laid end to
// end and cut into equal contiguous ranges, one per pair.  A range that starts
// inside a tile is the pair's first unit: it writes its fp32 partial tile to the
// workspace and publishes a flag.  The unit that holds the start of a tile is the
// last unit of its pair: it waits (bounded) for the flags of the following pairs
// whose ranges cover the rest of the tile, adds their partials in K order (a
// fixed order, so results are deterministic), and runs the bias/cast epilogue.
// Flags carry a generation number kept in the workspace and advanced by the
// last CTA of each launch, so flags of an earlier or aborted launch never match.
#include <algorithm>
#include <atomic>

#include "svdq_common.cuh"

namespace svdq {
namespace {

constexpr int BM = 128;          // rows per CTA (the pair tile is 2*BM)
constexpr int BN = 256;          // columns per tile
constexpr int BN_HALF = BN / 2;  // W rows staged per CTA
constexpr int KB = 128;          // bytes of K per operand stage row (64 fp16/bf16)
constexpr int STAGES = 6;
constexpr int A_BYTES = BM * KB;       // 16 KiB
constexpr int B_BYTES = BN_HALF * KB;  // 16 KiB
constexpr int AB_BYTES = A_BYTES + B_BYTES;
constexpr int NUM_THREADS = 384;
constexpr int NUM_ACC = 2;             // TMEM accumulators (tile double buffering)
constexpr int TMEM_COLS = NUM_ACC * BN;
constexpr int EPI_COLS = BN / 2;       // columns per epilogue warpgroup
static_assert(A_BYTES % 1024 == 0 && B_BYTES % 1024 == 0, "operand tiles keep 1 KiB alignment for 128B swizzle");
static_assert(TMEM_COLS == 512, "TMEM allocation");

struct Barriers {
  uint64_t full[STAGES];       // used in the even CTA (both CTAs' loads count here)
  uint64_t empty[STAGES];
  uint64_t tmem_full[NUM_ACC];
  uint64_t tmem_empty[NUM_ACC];  // used in the even CTA (16 arrivals: 8 warps per CTA)
  uint64_t mma_done;
  uint64_t part_done;          // epilogue warps of this CTA have written a tail partial (8 arrivals)
  uint32_t tmem_base;
  int abort_flag;
};

constexpr size_t SMEM_BYTES = (size_t)STAGES * AB_BYTES + sizeof(Barriers) + 1024;

// One GEMM of a launch.  A grouped launch runs up to kMaxProblems GEMMs that share M, K_pad and
// R2 (layers reading the same activations) over one persistent grid: their tiles are numbered
// one after the other, problem by problem.
constexpr int kMaxProblems = 4;
struct GemmProblem {
  const __nv_bfloat16* bias;
  void* out;
  int64_t ldo;
  const void* aux;  // epilogue operand z [M, N] in out's dtype (row stride ld_aux); the operation is
                    // the kernel's EPI template parameter, shared by the problems of a launch
  int64_t ld_aux;
  int N;
  int num_n_blocks;
  int tile_start;   // index of the problem's first tile
};

struct TmaSet {  // tensor maps of each problem: a16, w16, mid_hl, up_hl
  CUtensorMap a[kMaxProblems], w[kMaxProblems], mid[kMaxProblems], up[kMaxProblems];
};

struct GemmArgs {
  GemmProblem prob[kMaxProblems];
  int num_problems;
  int M;
  int n_k;   // K_pad / 64 residual stages
  int n_lr;  // R2 / 64 low-rank stages
  int num_m_blocks;  // pair tiles: 256 rows x 256 columns
  int iters;       // K iterations of one tile: n_k + n_lr
  int dp_tiles;    // tiles [0, dp_tiles) are computed whole, round-robin over the pairs
  int tail_len;    // K iterations per pair in the split tail
  int tail_total;  // (num_tiles - dp_tiles) * iters; 0 = no split tail
  float* partial;  // [2 * pairs][BM * BN] fp32 partial tiles of the split tail
  uint32_t* sync;  // [0] generation, [1] CTAs done, [2 + 2 * pair + rank] partial-ready flags
  int* err;
};

// Workspace of the split tail: sync words, then one fp32 partial tile per CTA.
constexpr size_t kPartialFloats = (size_t)BM * BN;
inline size_t sync_bytes(int max_pairs) { return ((size_t)(2 + 2 * max_pairs) * 4 + 1023) / 1024 * 1024; }
inline size_t workspace_bytes_for(int max_pairs) {
  return sync_bytes(max_pairs) + (size_t)2 * max_pairs * kPartialFloats * sizeof(float);
}
constexpr int kMaxParts = 4;       // a tail tile is cut into at most this many K ranges
constexpr int kMinSplitIters = 8;  // and no range is shorter than this many K iterations

// Wait sites recorded in the device error word.
enum : int {
  kWaitProdEmpty = 0x101,
  kWaitMmaFull = 0x201,
  kWaitMmaTmemEmpty = 0x202,
  kWaitMmaDone = 0x203,
  kWaitEpiTmemFull = 0x301,
  kWaitEpiPartial = 0x302,   // the owner of a split tile waited for a partial
  kWaitEpiPartDone = 0x303,  // a CTA waited for its own epilogue warps' partial stores
};

constexpr uint32_t kFmtF16 = 0;  // kind::f16 format code for fp16

// Epilogue operations: the linear's output y (accumulator + bias) combined with an operand z of
// the output's shape and dtype, in the order of the elementwise torch ops they replace.  With bf16
// output every value torch would store (y, the activation) is rounded to bf16 first, so the result
// is the unfused sequence's.
enum : int {
  kEpiNone = 0,
  kEpiAdd = 1,         // z + y                  (residual add)
  kEpiSigmoidMul = 2,  // z * sigmoid(y)         (attention output gated by to_gate)
  kEpiSiluMul = 3,     // silu(z) * y            (gated MLP: z = ff.gate output, y = ff.up)
};

// Two values rounded to bf16 and widened back, through the packed two-value conversion and
// integer shifts.  The XU pipe also issues the activations' ex2 and reciprocal; with the
// single-value conversion and its way back instead, ncu counted XU instructions at 14.7% of peak
// against 9.0% in the sigmoid epilogue, and that launch ran 8 us longer (M 4352, N 6144, K 6144).
__device__ __forceinline__ float2 bf16r2(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  const uint32_t w = *reinterpret_cast<const uint32_t*>(&h);
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}

// sigmoid(v) or silu(v) in fp32 as torch evaluates them (expf, IEEE division).
template <int EPI>
__device__ __forceinline__ float act_exact(float v) {
  return EPI == kEpiSigmoidMul ? 1.0f / (1.0f + expf(-v)) : v / (1.0f + expf(-v));
}
// e^x for |x| <= 64, to a few ulp: Cody-Waite style range reduction to base 2 (J.-M. Muller,
// "Elementary Functions", ch. 11), with the product x * log2(e) formed exactly as hi + lo by an FMA
// against log2(e) split into a float and its float remainder.  2^hi comes from the ex2.approx
// instruction and 2^lo as 1 + lo * ln 2: |lo| < 2^-17, so the dropped quadratic term is below
// 2^-35 relative.  The plain ex2.approx(x * log2 e) loses up to |x| / 2 ulp to the rounding of that
// product, which epi_act8_fast below would have to cover with a far wider fallback window.
__device__ __forceinline__ float exp_split(float x) {
  constexpr float kLog2e = 1.44269502162933349609375f;  // float(log2 e)
  constexpr float kLog2eLo = 1.925963033500011e-08f;    // log2 e - kLog2e
  constexpr float kLn2 = 0.693147182464599609375f;
  const float hi = x * kLog2e;
  const float lo = fmaf(x, kLog2e, -hi) + x * kLog2eLo;
  float p;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(p) : "f"(hi));
  return fmaf(p, lo * kLn2, p);
}
// The operation on 8 outputs (the kernel is instantiated per operation, so a launch without one
// carries no epilogue-operand code).  fp32 output evaluates the activation exactly, out of line.
template <bool F32, int EPI>
__device__ __noinline__ void epi_act8_f32(float (&v)[8], const float (&z)[8]) {
#pragma unroll
  for (int e = 0; e < 8; ++e)
    v[e] = EPI == kEpiSigmoidMul ? z[e] * act_exact<EPI>(v[e]) : act_exact<EPI>(z[e]) * v[e];
}
template <bool F32, int EPI>
__device__ __forceinline__ void epi_apply(float (&v)[8], const float (&z)[8]) {
  if constexpr (EPI == kEpiAdd) {
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      const float2 y = F32 ? make_float2(v[e], v[e + 1]) : bf16r2(v[e], v[e + 1]);
      v[e] = z[e] + y.x;
      v[e + 1] = z[e + 1] + y.y;
    }
  } else {
    static_assert(F32, "bf16 activations go through epi_act8_bf16");
    epi_act8_f32<F32, EPI>(v, z);
  }
}
// bf16 output of an activation epilogue on 8 outputs y (accumulator + bias) and their operand
// words zw: the 8 results packed, and a flag set if any of them needs the exact path.
// The activation comes from exp_split and the approximate reciprocal.  For |v| <= 64 that fp32
// value differs from the exact path's by at most ~17 ulp (ex2.approx and the reciprocal 2^-22
// relative each, four roundings, and the exact path's own expf error), so one whose low 16 bits
// lie more than 32 ulp from the bf16 rounding midpoint 0x8000 rounds to the same bf16 value; the
// others (about 0.1% of inputs), and |v| > 64 or NaN, are flagged.  tests/test_gpu_epilogue.py
// checks all 65536 bf16 inputs against torch.
// Out of line, with every value in registers (no stack frame): a thread's 128 columns per tile
// share one copy of the code, and the exact path is a separate call that ~1% of calls make.  The
// same function inlined (16 copies per thread) made the sigmoid and SiLU launches 4-6% slower
// (M 4352, K 6144, N 6144 and 16384, alternated in one process).
struct Act8 {
  uint4 w;        // 8 packed bf16 results
  uint32_t slow;  // nonzero: some result needs the exact path
};
template <int EPI>
__device__ __noinline__ Act8 epi_act8_fast(float4 ya, float4 yb, uint4 zw) {
  const float y[8] = {ya.x, ya.y, ya.z, ya.w, yb.x, yb.y, yb.z, yb.w};
  const uint32_t zz[4] = {zw.x, zw.y, zw.z, zw.w};
  uint32_t w[4], slow = 0;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 zf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&zz[e]));
    const float2 yv = bf16r2(y[2 * e], y[2 * e + 1]);
    const float v[2] = {EPI == kEpiSigmoidMul ? yv.x : zf.x, EPI == kEpiSigmoidMul ? yv.y : zf.y};
    float sv[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float r = __fdividef(1.0f, 1.0f + exp_split(-v[h]));
      sv[h] = EPI == kEpiSigmoidMul ? r : v[h] * r;
      slow |= (uint32_t)(!(fabsf(v[h]) <= 64.0f) || (__float_as_uint(sv[h]) & 0xFFFFu) - 0x7FE0u <= 0x40u);
    }
    const float2 a = bf16r2(sv[0], sv[1]);
    const float o0 = EPI == kEpiSigmoidMul ? zf.x * a.x : a.x * yv.x;
    const float o1 = EPI == kEpiSigmoidMul ? zf.y * a.y : a.y * yv.y;
    __nv_bfloat162 hh = __floats2bfloat162_rn(o0, o1);
    w[e] = *reinterpret_cast<uint32_t*>(&hh);
  }
  return Act8{make_uint4(w[0], w[1], w[2], w[3]), slow};
}
// The same from the exact activation, for the calls epi_act8_fast flagged (on its unflagged
// outputs both give the same bf16, so all eight are recomputed).
template <int EPI>
__device__ __noinline__ uint4 epi_act8_exact(float4 ya, float4 yb, uint4 zw) {
  const float y[8] = {ya.x, ya.y, ya.z, ya.w, yb.x, yb.y, yb.z, yb.w};
  const uint32_t zz[4] = {zw.x, zw.y, zw.z, zw.w};
  uint32_t w[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 zf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&zz[e]));
    const float2 yv = bf16r2(y[2 * e], y[2 * e + 1]);
    const float2 a = EPI == kEpiSigmoidMul ? bf16r2(act_exact<EPI>(yv.x), act_exact<EPI>(yv.y))
                                           : bf16r2(act_exact<EPI>(zf.x), act_exact<EPI>(zf.y));
    const float o0 = EPI == kEpiSigmoidMul ? zf.x * a.x : a.x * yv.x;
    const float o1 = EPI == kEpiSigmoidMul ? zf.y * a.y : a.y * yv.y;
    __nv_bfloat162 hh = __floats2bfloat162_rn(o0, o1);
    w[e] = *reinterpret_cast<uint32_t*>(&hh);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}
template <int EPI>
__device__ __forceinline__ uint4 epi_act8_bf16(float4 ya, float4 yb, uint4 zw) {
  const Act8 r = epi_act8_fast<EPI>(ya, yb, zw);
  return r.slow ? epi_act8_exact<EPI>(ya, yb, zw) : r.w;
}
template <int EPI>
__device__ __forceinline__ uint2 epi_act4_bf16(float4 ya, uint2 zw) {
  const uint4 r = epi_act8_bf16<EPI>(ya, make_float4(0.f, 0.f, 0.f, 0.f), make_uint4(zw.x, zw.y, 0u, 0u));
  return make_uint2(r.x, r.y);
}

__device__ __forceinline__ void advance(int& idx, uint32_t& phase, int n) {
  if (++idx == n) {
    idx = 0;
    phase ^= 1u;
  }
}

// Tile t -> (row block, column block).  Row blocks advance along N in groups of kGroupM, so the
// tiles live at one time share about 8 A slabs and a few W slabs, which stay in L2: at
// M4096 N16384 K6144 this reads 570 MB of DRAM against 707 MB for plain column-major order
// (groups of 4: 989 MB, groups of 12: 633 MB and 2% slower).
constexpr int kGroupM = 8;

// Problem of global tile t, and t's index within it.  Unrolled over the problems so that every
// parameter access has a constant offset.
__device__ __forceinline__ int tile_problem(const GemmArgs& a, int& t) {
  int p = 0;
#pragma unroll
  for (int i = 1; i < kMaxProblems; ++i)
    if (i < a.num_problems && t >= a.prob[i].tile_start) p = i;
  int start = 0;
#pragma unroll
  for (int i = 1; i < kMaxProblems; ++i)
    if (i == p) start = a.prob[i].tile_start;
  t -= start;
  return p;
}
__device__ __forceinline__ GemmProblem get_problem(const GemmArgs& a, int p) {
  GemmProblem r = a.prob[0];
#pragma unroll
  for (int i = 1; i < kMaxProblems; ++i)
    if (i == p) r = a.prob[i];
  return r;
}
__device__ __forceinline__ const CUtensorMap* pick_map(const CUtensorMap (&m)[kMaxProblems], int p) {
  const CUtensorMap* r = &m[0];
#pragma unroll
  for (int i = 1; i < kMaxProblems; ++i)
    if (i == p) r = &m[i];
  return r;
}

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& mb, int& nb) {
  const int per_group = kGroupM * num_n;
  const int first_m = (t / per_group) * kGroupM;
  const int r = t % per_group;
  const int gm = min(num_m - first_m, kGroupM);
  mb = first_m + r % gm;
  nb = r / gm;
}

// The units of one pair, in order: whole tiles pair, pair + pairs, ... below
// dp_tiles, then the pieces of its tail range [pair * tail_len, +tail_len),
// cut at tile boundaries.  A unit is (tile, K iterations [k0, k1)).
struct Walk {
  int j, g, gend;
};
__device__ __forceinline__ void walk_init(Walk& w, const GemmArgs& a, int pair) {
  w.j = 0;
  w.g = a.tail_total > 0 ? min(pair * a.tail_len, a.tail_total) : 0;
  w.gend = a.tail_total > 0 ? min(w.g + a.tail_len, a.tail_total) : 0;
}
__device__ __forceinline__ bool walk_next(Walk& w, const GemmArgs& a, int pair, int num_pairs, int& t, int& k0,
                                          int& k1) {
  const int td = pair + w.j * num_pairs;
  if (td < a.dp_tiles) {
    ++w.j;
    t = td;
    k0 = 0;
    k1 = a.iters;
    return true;
  }
  if (w.g >= w.gend) return false;
  const int tt = w.g / a.iters;
  k0 = w.g - tt * a.iters;
  k1 = min(a.iters, k0 + (w.gend - w.g));
  t = a.dp_tiles + tt;
  w.g += k1 - k0;
  return true;
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void mbar_arrive_local(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Element (row, col) of a CTA's partial tile: 4-column groups outermost, so the
// 32 lanes of a warp (32 consecutive rows) touch 512 contiguous bytes.
__device__ __forceinline__ size_t part_index(int row, int col) {
  return ((size_t)(col >> 2) * BM + row) * 4 + (col & 3);
}

// An owner streams the partials it adds through the operand ring, idle by then
// (its unit is the pair's last): per epilogue warp kPartSlots groups of 8 x 512
// bytes, one group = one 32-column chunk of one partial for the warp's 32 rows.
constexpr int kPartSlots = 6;
constexpr uint32_t kPartWarpBytes = kPartSlots * 8 * 512;
static_assert(8 * kPartWarpBytes <= (uint32_t)STAGES * AB_BYTES, "partial staging fits the operand ring");

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ float4 ld_shared_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}

template <bool OUT_F32, int EPI>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    linear_gemm_kernel(const __grid_constant__ TmaSet maps, const __grid_constant__ GemmArgs args) {
  constexpr int kOutBytes = OUT_F32 ? 4 : 2;
  constexpr int kAuxWords = 32 * kOutBytes / 16;  // 16-byte words of z per 32-column chunk
  constexpr int kAuxBufs = OUT_F32 ? 1 : 2;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw_addr & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  const uint32_t smem_base = raw_addr + pad;
  Barriers* bars = reinterpret_cast<Barriers*>(smem + (size_t)STAGES * AB_BYTES);
  volatile int* abort_flag = &bars->abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 = even CTA (MMA issuer), 1 = its pair
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;

  auto full_bar = [&](int s) { return smem_u32(&bars->full[s]); };
  auto empty_bar = [&](int s) { return smem_u32(&bars->empty[s]); };
  auto tm_full = [&](int b) { return smem_u32(&bars->tmem_full[b]); };
  auto tm_empty = [&](int b) { return smem_u32(&bars->tmem_empty[b]); };
  auto stage_a = [&](int s) { return smem_base + (uint32_t)(s * AB_BYTES); };
  auto stage_b = [&](int s) { return smem_base + (uint32_t)(s * AB_BYTES + A_BYTES); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);   // the even CTA's producer arrives (with both CTAs' bytes)
      mbar_init(empty_bar(s), 1);  // MMA commit
    }
    for (int b = 0; b < NUM_ACC; ++b) {
      mbar_init(tm_full(b), 1);
      mbar_init(tm_empty(b), 16);  // epilogue warps of both CTAs
    }
    mbar_init(smem_u32(&bars->mma_done), 1);
    mbar_init(smem_u32(&bars->part_done), 8);  // one arrival per epilogue warp
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
#pragma unroll
    for (int i = 0; i < kMaxProblems; ++i) {
      if (i < args.num_problems) {
        prefetch_tma_desc(&maps.a[i]);
        prefetch_tma_desc(&maps.w[i]);
        if (args.n_lr > 0) {
          prefetch_tma_desc(&maps.mid[i]);
          prefetch_tma_desc(&maps.up[i]);
        }
      }
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(&bars->tmem_base), TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers are initialised before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;
  // everything above touches no memory an earlier kernel writes; operands are read from here on
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer (both CTAs)
      int stage = 0;
      uint32_t phase = 0;
      uint32_t filled = 0, par = 0;
      bool ok = true;
      Walk wk;
      walk_init(wk, args, pair);
      int t, k0, k1;
      while (ok && walk_next(wk, args, pair, num_pairs, t, k0, k1)) {
        int tp = t;
        const int p = tile_problem(args, tp);
        const GemmProblem P = get_problem(args, p);
        const CUtensorMap* tm_a = pick_map(maps.a, p);
        const CUtensorMap* tm_w = pick_map(maps.w, p);
        const CUtensorMap* tm_mid = pick_map(maps.mid, p);
        const CUtensorMap* tm_up = pick_map(maps.up, p);
        int mb, nb;
        tile_coords(tp, args.num_m_blocks, P.num_n_blocks, mb, nb);
        const int m0 = mb * (2 * BM) + (int)rank * BM;
        const int n0 = nb * BN + (int)rank * BN_HALF;
        for (int s = k0; ok && s < k1; ++s) {
          if (!(ok = mbar_wait<true>(empty_bar(stage), phase ^ 1u, abort_flag, args.err, kWaitProdEmpty))) break;
          const uint32_t full_c = mapa_shared(full_bar(stage), 0);
          if (leader) mbar_arrive_expect_tx(full_bar(stage), 2 * AB_BYTES);
          if (s < args.n_k) {
            tma_load_2d_pair(stage_a(stage), tm_a, full_c, s * 64, m0);
            tma_load_2d_pair(stage_b(stage), tm_w, full_c, s * 64, n0);
          } else {
            tma_load_2d_pair(stage_a(stage), tm_mid, full_c, (s - args.n_k) * 64, m0);
            tma_load_2d_pair(stage_b(stage), tm_up, full_c, (s - args.n_k) * 64, n0);
          }
          filled |= 1u << stage;
          par = (par & ~(1u << stage)) | (phase << stage);
          advance(stage, phase, STAGES);
        }
      }
      if (!ok && leader) {
        // let copies already in flight land before the CTA exits
        for (int s = 0; s < STAGES; ++s)
          if (filled & (1u << s)) mbar_wait_drain(full_bar(s), (par >> s) & 1u, 100000000ull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------------------------------------ MMA issuer (even CTA)
      const uint32_t idesc_f16 = make_idesc(kFmtF16, kFmtF16, 2 * BM, BN);
      const uint32_t idesc_bf16 = make_idesc(kFmtBF16, kFmtBF16, 2 * BM, BN);
      int stage = 0, tb = 0;
      uint32_t phase = 0, tb_ph = 0;
      bool ok = true;
      Walk wk;
      walk_init(wk, args, pair);
      int t, k0, k1;
      while (ok && walk_next(wk, args, pair, num_pairs, t, k0, k1)) {
        if (!(ok = mbar_wait<true>(tm_empty(tb), tb_ph ^ 1u, abort_flag, args.err, kWaitMmaTmemEmpty))) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(tb * BN);
        for (int s = k0; ok && s < k1; ++s) {
          if (!(ok = mbar_wait<true>(full_bar(stage), phase, abort_flag, args.err, kWaitMmaFull))) break;
          tc_fence_after();
          const uint64_t da = desc_k_sw128(stage_a(stage));
          const uint64_t db = desc_k_sw128(stage_b(stage));
          const uint32_t idesc = s < args.n_k ? idesc_f16 : idesc_bf16;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)  // 4 x K=16 = 128 bytes
            umma_f16_pair(d, da + (uint64_t)(kk * 2), db + (uint64_t)(kk * 2), idesc, (s > k0 || kk > 0) ? 1u : 0u);
          umma_commit_pair(empty_bar(stage));
          advance(stage, phase, STAGES);
        }
        if (!ok) break;
        umma_commit_pair(tm_full(tb));
        advance(tb, tb_ph, NUM_ACC);
      }
      // all issued MMAs must finish before either CTA releases TMEM or exits
      umma_commit_pair_local(smem_u32(&bars->mma_done));
      if (!mbar_wait_drain(smem_u32(&bars->mma_done), 0, 1000000000ull)) {
        *abort_flag = 1;
        atomicCAS(args.err, 0, kWaitMmaDone);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int ew = warp - 4;
    const int q = warp & 3;                 // TMEM lane quarter this warp may access
    const int col0 = (ew >> 2) * EPI_COLS;  // warpgroup's column half
    const int row = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    // flag value of this launch: flags of earlier launches hold older generations
    const uint32_t epoch = args.tail_total > 0 ? *reinterpret_cast<volatile uint32_t*>(args.sync) + 1u : 0u;
    int tb = 0;
    uint32_t tb_ph = 0;
    bool ok = true;
    Walk wk;
    walk_init(wk, args, pair);
    int t, k0, k1;
    while (ok && walk_next(wk, args, pair, num_pairs, t, k0, k1)) {
      int tp = t;
      const GemmProblem P = get_problem(args, tile_problem(args, tp));
      int mb, nb;
      tile_coords(tp, args.num_m_blocks, P.num_n_blocks, mb, nb);
      const int m0 = mb * (2 * BM) + (int)rank * BM;
      const int n0 = nb * BN;
      const bool contrib = k0 > 0;  // a later piece of a split tile: hand the partial to its owner
      int n_parts = 0;              // owner of a split tile: partials of pairs pair+1 .. pair+n_parts
      if (k0 == 0 && k1 < args.iters) {
        const int tile_end = (t - args.dp_tiles + 1) * args.iters;
        for (int c = pair + 1; c < num_pairs && c * args.tail_len < tile_end; ++c) ++n_parts;
      }
      // bias of the warpgroup's 128 columns: lane l < 16 holds columns 8l .. 8l+7, loaded
      // before the accumulator wait so its latency hides behind the MMAs
      uint4 bias_lane = make_uint4(0u, 0u, 0u, 0u);
      if (P.bias && !contrib && lane < 16 && n0 + col0 + 8 * lane < P.N)
        bias_lane = *reinterpret_cast<const uint4*>(P.bias + n0 + col0 + 8 * lane);
      // epilogue operand: the lane's row, 32 columns per chunk; bf16 one chunk ahead (the first
      // one before the accumulator wait), fp32 (twice the registers) at the chunk's start;
      // streamed with an evict-first hint, it is read once
      const int grow = m0 + row;
      const bool use_aux = EPI != kEpiNone && !contrib;
      const uint8_t* aux_row = static_cast<const uint8_t*>(P.aux) + (size_t)grow * P.ld_aux * kOutBytes;
      uint4 ax[EPI != kEpiNone ? kAuxBufs : 1][kAuxWords];
      auto load_aux = [&](int c, uint4 (&d)[kAuxWords]) {
#pragma unroll
        for (int i = 0; i < kAuxWords; ++i) {
          const int n = n0 + col0 + c * 32 + i * (16 / kOutBytes);
          d[i] = (grow < args.M && n < P.N) ? __ldcs(reinterpret_cast<const uint4*>(aux_row + (size_t)n * kOutBytes))
                                               : make_uint4(0u, 0u, 0u, 0u);
        }
      };
      if (use_aux && kAuxBufs == 2) load_aux(0, ax[0]);
      if (!(ok = mbar_wait<true>(tm_full(tb), tb_ph, abort_flag, args.err, kWaitEpiTmemFull))) break;
      tc_fence_after();
      if (n_parts > 0) {
        // lane 0 waits for each flag (bounded); then every lane acquires it itself
        int good = 1;
        if (lane == 0) {
          for (int c = 1; c <= n_parts && good; ++c) {
            const uint32_t* f = args.sync + 2 + 2 * (pair + c) + rank;
            if (ld_acquire_gpu(f) == epoch) continue;
            const unsigned long long t0 = globaltimer();
            while (ld_acquire_gpu(f) != epoch) {
              if (*abort_flag) { good = 0; break; }
              if (globaltimer() - t0 > kWaitLimitNs) {
                *abort_flag = 1;
                atomicCAS(args.err, 0, kWaitEpiPartial);
                good = 0;
                break;
              }
            }
          }
        }
        good = __shfl_sync(0xffffffffu, good, 0);
        if (!(ok = good != 0)) break;
        for (int c = 1; c <= n_parts; ++c) (void)ld_acquire_gpu(args.sync + 2 + 2 * (pair + c) + rank);
      }
      // owner: groups (chunk c, partial pc) in the order they are added, kPartSlots in flight;
      // each lane copies and later reads only its own 16-byte pieces (no cross-lane hazards)
      const uint32_t wreg = smem_base + (uint32_t)ew * kPartWarpBytes;
      const int n_groups = 4 * n_parts;
      auto issue_group = [&](int g) {
        if (g < n_groups) {
          const int c = g / n_parts, pc = g - c * n_parts + 1;
          const float* src = args.partial + (size_t)(2 * (pair + pc) + (int)rank) * kPartialFloats +
                             part_index(row, col0 + c * 32);
          const uint32_t dst = wreg + (uint32_t)(g % kPartSlots) * (8 * 512) + (uint32_t)lane * 16;
#pragma unroll
          for (int i = 0; i < 8; ++i) cp_async16(dst + (uint32_t)i * 512, src + (size_t)i * 4 * BM);
        }
        cp_async_commit();
      };
      if (n_parts > 0)
        for (int g = 0; g < kPartSlots; ++g) issue_group(g);
      const uint32_t taddr = tmem_base + lane_off + (uint32_t)(tb * BN + col0);
      const int64_t rbase = (int64_t)grow * P.ldo;
      uint32_t va[32], vb[32];
      tmem_ld32(taddr, va);
#pragma unroll
      for (int c = 0; c < EPI_COLS / 32; ++c) {
        uint32_t (&cur)[32] = (c & 1) ? vb : va;
        uint32_t (&nxt)[32] = (c & 1) ? va : vb;
        if (use_aux && kAuxBufs == 1) load_aux(c, ax[0]);
        tmem_ld_wait_regs(cur);
        if (c + 1 < EPI_COLS / 32) {
          tmem_ld32(taddr + (uint32_t)((c + 1) * 32), nxt);
        } else {
          // the whole accumulator slice is in registers: hand TMEM back to the MMA warp
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(mapa_shared(tm_empty(tb), 0));
        }
        if (use_aux && kAuxBufs == 2 && c + 1 < EPI_COLS / 32) load_aux(c + 1, ax[(c + 1) % kAuxBufs]);
        const int cc = col0 + c * 32;  // tile column of cur[0]
        if (contrib) {
          float4* slot = reinterpret_cast<float4*>(args.partial + (size_t)(2 * pair + (int)rank) * kPartialFloats);
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            __stcg(slot + part_index(row, cc + i) / 4, make_float4(__uint_as_float(cur[i]), __uint_as_float(cur[i + 1]),
                                                                   __uint_as_float(cur[i + 2]), __uint_as_float(cur[i + 3])));
          continue;
        }
        // owner of a split tile: add the other ranges' partials in K order
        for (int pc = 1; pc <= n_parts; ++pc) {
          const int g = c * n_parts + pc - 1;
          cp_async_wait<kPartSlots - 1>();  // groups up to g have landed
          const uint32_t sl = wreg + (uint32_t)(g % kPartSlots) * (8 * 512) + (uint32_t)lane * 16;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 pv = ld_shared_f4(sl + (uint32_t)i * 512);
            cur[4 * i] = __float_as_uint(__uint_as_float(cur[4 * i]) + pv.x);
            cur[4 * i + 1] = __float_as_uint(__uint_as_float(cur[4 * i + 1]) + pv.y);
            cur[4 * i + 2] = __float_as_uint(__uint_as_float(cur[4 * i + 2]) + pv.z);
            cur[4 * i + 3] = __float_as_uint(__uint_as_float(cur[4 * i + 3]) + pv.w);
          }
          issue_group(g + kPartSlots);  // reuses the slot just read (its values are in registers)
        }
        const int nc = n0 + cc;
        uint32_t bw[4][4];  // bias words of this chunk's four 8-column groups
#pragma unroll
        for (int ii = 0; ii < 4; ++ii) {
          bw[ii][0] = __shfl_sync(0xffffffffu, bias_lane.x, c * 4 + ii);
          bw[ii][1] = __shfl_sync(0xffffffffu, bias_lane.y, c * 4 + ii);
          bw[ii][2] = __shfl_sync(0xffffffffu, bias_lane.z, c * 4 + ii);
          bw[ii][3] = __shfl_sync(0xffffffffu, bias_lane.w, c * 4 + ii);
        }
        if (grow < args.M) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            const int n = nc + i;
            if (n < P.N) {
              float v[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(cur[i + e]);
              if (P.bias) {
                const __nv_bfloat162* bb = reinterpret_cast<const __nv_bfloat162*>(bw[i / 8]);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float2 f = __bfloat1622float2(bb[e]);
                  v[2 * e] += f.x;
                  v[2 * e + 1] += f.y;
                }
              }
              if constexpr (!OUT_F32 && (EPI == kEpiSigmoidMul || EPI == kEpiSiluMul)) {
                if (use_aux) {
                  *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(P.out) + rbase + n) =
                      epi_act8_bf16<EPI>(make_float4(v[0], v[1], v[2], v[3]), make_float4(v[4], v[5], v[6], v[7]),
                                         ax[c % kAuxBufs][i / 8]);
                  continue;
                }
              } else if constexpr (EPI != kEpiNone) {
               if (use_aux) {
                float z[8];
                if constexpr (OUT_F32) {
                  const uint4 z0 = ax[c % kAuxBufs][2 * (i / 8)], z1 = ax[c % kAuxBufs][2 * (i / 8) + 1];
                  z[0] = __uint_as_float(z0.x), z[1] = __uint_as_float(z0.y);
                  z[2] = __uint_as_float(z0.z), z[3] = __uint_as_float(z0.w);
                  z[4] = __uint_as_float(z1.x), z[5] = __uint_as_float(z1.y);
                  z[6] = __uint_as_float(z1.z), z[7] = __uint_as_float(z1.w);
                } else {
                  const uint4 zw = ax[c % kAuxBufs][i / 8];
                  const uint32_t zz[4] = {zw.x, zw.y, zw.z, zw.w};
#pragma unroll
                  for (int e = 0; e < 4; ++e) {
                    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&zz[e]));
                    z[2 * e] = f.x;
                    z[2 * e + 1] = f.y;
                  }
                }
                epi_apply<OUT_F32, EPI>(v, z);
               }
              }
              if constexpr (OUT_F32) {
                float4* o = reinterpret_cast<float4*>(static_cast<float*>(P.out) + rbase + n);
                o[0] = make_float4(v[0], v[1], v[2], v[3]);
                o[1] = make_float4(v[4], v[5], v[6], v[7]);
              } else {
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
                  w[e] = *reinterpret_cast<uint32_t*>(&h);
                }
                *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(P.out) + rbase + n) =
                    make_uint4(w[0], w[1], w[2], w[3]);
              }
            }
          }
        }
      }
      if (contrib) {
        // publish the partial: each warp's arrival (release at CTA scope) orders its stores
        // before the publishing thread's acquire, whose GPU-scope release then covers them
        __syncwarp();
        if (lane == 0) mbar_arrive_local(smem_u32(&bars->part_done));
        int good = 1;
        if (ew == 0) {
          if (lane == 0) {
            if (mbar_wait<false>(smem_u32(&bars->part_done), 0, abort_flag, args.err, kWaitEpiPartDone)) {
              __threadfence();
              st_release_gpu(args.sync + 2 + 2 * pair + rank, epoch);
            } else {
              good = 0;
            }
          }
          good = __shfl_sync(0xffffffffu, good, 0);
        }
        if (!(ok = good != 0)) break;
      }
      advance(tb, tb_ph, NUM_ACC);
    }
  }

  // Neither CTA may exit or release TMEM while the pair's MMAs can still touch
  // its shared memory or TMEM; every role above has left its loop (all waits
  // are bounded) and the even CTA's MMA warp has drained its MMAs.
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
  if (args.tail_total > 0 && threadIdx.x == 0) {
    // the last CTA of the launch advances the generation (every CTA has read it by now)
    __threadfence();
    if (atomicAdd(args.sync + 1, 1u) == gridDim.x - 1) {
      args.sync[1] = 0;
      args.sync[0] = args.sync[0] + 1u;
      __threadfence();
    }
  }
}

}  // namespace

// Pairs of this kernel that can be resident at once on the current device.  The
// split tail's owners wait for other pairs, so its grid never exceeds this.
int max_resident_pairs(const void* kern) {
  static std::atomic<int> cache[64];  // per device; concurrent fillers store the same value
  int dev = 0;
  cudaGetDevice(&dev);
  const int fallback = num_sms() / 2;
  if (dev < 0 || dev >= 64) return fallback;
  int c = cache[dev].load(std::memory_order_relaxed);
  if (c == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * fallback, 1, 1);
    cfg.blockDim = dim3(NUM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
      (void)cudaGetLastError();
      n = fallback;
    }
    c = n < fallback ? n : fallback;
    cache[dev].store(c, std::memory_order_relaxed);
  }
  return c;
}

struct Schedule {
  int pairs, dp_tiles, tail_len, tail_total;
};

// Whole tiles round-robin; a last partial wave filling at most 11/20 of the pairs
// is split into equal K ranges when the workspace allows (see the kernel comment).
// A split tail costs about three tile epilogues of fixed time (partial stores,
// flag hand-off, partial loads), so fuller last waves stay whole: measured on
// B200 at M 4352, K 6144, a tail of 0.38 of a wave ran 8% faster split, one of
// 0.70 ran 1% slower.
Schedule plan_schedule(int tiles, int iters, int max_pairs, bool can_split) {
  Schedule s{tiles < max_pairs ? tiles : max_pairs, tiles, 0, 0};
  if (!can_split || tiles <= 0) return s;
  const int full = tiles / max_pairs, tail = tiles - full * max_pairs;
  if (tail == 0 || tail * 20 > max_pairs * 11) return s;
  const int tail_total = tail * iters;
  int len = (tail_total + max_pairs - 1) / max_pairs;
  len = std::max(len, std::max(kMinSplitIters, (iters + kMaxParts - 1) / kMaxParts));
  if (len >= iters) return s;
  s.dp_tiles = full * max_pairs;
  s.tail_len = len;
  s.tail_total = tail_total;
  s.pairs = full > 0 ? max_pairs : (tail_total + len - 1) / len;
  return s;
}

// Validates a group of GEMMs sharing M, K_pad and R2 and launches them as one persistent grid
// (a single problem is the plain GEMM).
int launch_linear_gemm_group(const svdq_gemm_problem* probs, int np, int R2, int out_dtype, int M, int K_pad,
                             void* workspace, size_t workspace_bytes, cudaStream_t stream, const char* who) {
  const std::string w(who);
  if (!probs || np < 1 || np > kMaxProblems)
    return set_error(SVDQ_ERR_INVALID_ARGUMENT, w + ": 1 to 4 problems per launch");
  if (!(M >= 0 && K_pad > 0)) return set_error(SVDQ_ERR_INVALID_ARGUMENT, w + ": bad M/K_pad");
  if (K_pad % 64 != 0) return set_error(SVDQ_ERR_INVALID_ARGUMENT, w + ": K_pad must be a multiple of 64");
  if (!(R2 >= 0 && R2 % 64 == 0)) return set_error(SVDQ_ERR_INVALID_ARGUMENT, w + ": R2 must be a multiple of 64");
  if (!(out_dtype == SVDQ_BF16 || out_dtype == SVDQ_FP32))
    return set_error(SVDQ_ERR_INVALID_ARGUMENT, w + ": out_dtype must be bf16 or fp32");
  for (int i = 0; i < np; ++i) {
    const svdq_gemm_problem& q = probs[i];
    const std::string wi = np > 1 ? w + " (problem " + std::to_string(i) + ")" : w;
    if (!(q.a16 && q.w16 && q.out)) return set_error(SVDQ_ERR_INVALID_ARGUMENT, wi + ": null operand pointer");
    if (!(q.N > 0 && q.N % 8 == 0 && q.ldo >= q.N && q.ldo % 8 == 0))
      return set_error(SVDQ_ERR_INVALID_ARGUMENT, wi + ": N and ldo must be positive multiples of 8, ldo >= N");
    if (R2 > 0 && !(q.mid_hl && q.up_hl))
      return set_error(SVDQ_ERR_INVALID_ARGUMENT, wi + ": mid_hl/up_hl are NULL");
    if (q.bias && (reinterpret_cast<uintptr_t>(q.bias) & 15u))
      return set_error(SVDQ_ERR_INVALID_ARGUMENT, wi + ": bias must be 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(q.out) & 15u)
      return set_error(SVDQ_ERR_INVALID_ARGUMENT, wi + ": out must be 16-byte aligned");
    if (!(q.epilogue >= kEpiNone && q.epilogue <= kEpiSiluMul))
      return set_error(SVDQ_ERR_INVALID_ARGUMENT, wi + ": unknown epilogue operation");
    if (q.epilogue != kEpiNone &&
        !(q.aux && (reinterpret_cast<uintptr_t>(q.aux) & 15u) == 0 && q.ld_aux >= q.N && q.ld_aux % 8 == 0))
      return set_error(SVDQ_ERR_INVALID_ARGUMENT,
                       wi + ": the epilogue operand must be non-null and 16-byte aligned, ld_aux >= N, ld_aux % 8 == 0");
  }
  if (M == 0) return SVDQ_OK;
  int* err = device_error_word();
  if (!err) return set_error(SVDQ_ERR_CUDA, w + ": device error word unavailable");

  TmaSet maps;
  GemmArgs a{};
  a.num_m_blocks = (M + 2 * BM - 1) / (2 * BM);
  int tiles = 0;
  for (int i = 0; i < np; ++i) {
    const svdq_gemm_problem& q = probs[i];
    int st;
    if ((st = make_tma_2d(&maps.a[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, q.a16, K_pad, M, (uint64_t)K_pad * 2, 64, BM,
                          CU_TENSOR_MAP_SWIZZLE_128B)))
      return st;
    if ((st = make_tma_2d(&maps.w[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, q.w16, K_pad, q.N, (uint64_t)K_pad * 2, 64,
                          BN_HALF, CU_TENSOR_MAP_SWIZZLE_128B)))
      return st;
    if (R2 > 0) {
      if ((st = make_tma_2d(&maps.mid[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, q.mid_hl, R2, M, (uint64_t)R2 * 2, 64,
                            BM, CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
      if ((st = make_tma_2d(&maps.up[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, q.up_hl, R2, q.N, (uint64_t)R2 * 2, 64,
                            BN_HALF, CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    } else {
      maps.mid[i] = maps.a[i];
      maps.up[i] = maps.w[i];
    }
    GemmProblem& g = a.prob[i];
    g.bias = static_cast<const __nv_bfloat16*>(q.bias);
    g.out = q.out;
    g.ldo = q.ldo;
    g.aux = q.epilogue != kEpiNone ? q.aux : nullptr;
    g.ld_aux = q.epilogue != kEpiNone ? q.ld_aux : 0;
    g.N = q.N;
    g.num_n_blocks = (q.N + BN - 1) / BN;
    g.tile_start = tiles;
    tiles += a.num_m_blocks * g.num_n_blocks;
  }
  for (int i = np; i < kMaxProblems; ++i) {  // never selected (tile_problem stops at num_problems)
    maps.a[i] = maps.a[0];
    maps.w[i] = maps.w[0];
    maps.mid[i] = maps.mid[0];
    maps.up[i] = maps.up[0];
    a.prob[i] = a.prob[0];
  }
  a.num_problems = np;
  a.M = M;
  a.n_k = K_pad / 64;
  a.n_lr = R2 / 64;
  a.iters = a.n_k + a.n_lr;
  a.err = err;
  const int epi = probs[0].epilogue;
  for (int i = 1; i < np; ++i)
    if (probs[i].epilogue != epi)
      return set_error(SVDQ_ERR_INVALID_ARGUMENT, w + ": every problem of a group takes the same epilogue operation");
  using Kern = void (*)(const TmaSet, const GemmArgs);
  static const Kern kerns[2][4] = {
      {linear_gemm_kernel<false, kEpiNone>, linear_gemm_kernel<false, kEpiAdd>,
       linear_gemm_kernel<false, kEpiSigmoidMul>, linear_gemm_kernel<false, kEpiSiluMul>},
      {linear_gemm_kernel<true, kEpiNone>, linear_gemm_kernel<true, kEpiAdd>,
       linear_gemm_kernel<true, kEpiSigmoidMul>, linear_gemm_kernel<true, kEpiSiluMul>}};
  const Kern kern = kerns[out_dtype == SVDQ_FP32 ? 1 : 0][epi];
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
  if (e != cudaSuccess) return check_cuda(e, (w + ": shared memory attribute").c_str());
  const int max_pairs = max_resident_pairs(reinterpret_cast<const void*>(kern));
  const bool can_split = workspace != nullptr && workspace_bytes >= workspace_bytes_for(num_sms() / 2) &&
                         (reinterpret_cast<uintptr_t>(workspace) & 255u) == 0;
  const Schedule sc = plan_schedule(tiles, a.iters, max_pairs, can_split);
  a.dp_tiles = sc.dp_tiles;
  a.tail_len = sc.tail_len;
  a.tail_total = sc.tail_total;
  a.sync = static_cast<uint32_t*>(workspace);
  a.partial = workspace ? reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + sync_bytes(num_sms() / 2))
                        : nullptr;
  const int pairs = sc.pairs;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, kern, maps, a);
  if (e != cudaSuccess) return check_cuda(e, (w + " launch").c_str());
  return check_launch((w + " launch").c_str());
}

int launch_linear_gemm(const void* a16, const void* w16, const void* mid_hl, const void* up_hl, int R2,
                       const void* bias, int epilogue, const void* aux, int64_t ld_aux, void* out, int out_dtype,
                       int64_t ldo, int M, int N, int K_pad, void* workspace, size_t workspace_bytes,
                       cudaStream_t stream, const char* who) {
  svdq_gemm_problem q{};
  q.a16 = a16;
  q.w16 = w16;
  q.mid_hl = mid_hl;
  q.up_hl = up_hl;
  q.bias = bias;
  q.epilogue = epilogue;
  q.aux = aux;
  q.ld_aux = ld_aux;
  q.out = out;
  q.ldo = ldo;
  q.N = N;
  if (N <= 0) return set_error(SVDQ_ERR_INVALID_ARGUMENT, std::string(who) + ": bad M/N/K_pad");
  return launch_linear_gemm_group(&q, 1, R2, out_dtype, M, K_pad, workspace, workspace_bytes, stream, who);
}

}  // namespace svdq

extern "C" int svdq_linear_gemm(const void* a16, const void* w16, const void* mid_hl, const void* up_hl, int R2,
                                const void* bias, void* out, int out_dtype, int64_t ldo, int M, int N, int K_pad,
                                cudaStream_t stream) {
  return svdq::launch_linear_gemm(a16, w16, mid_hl, up_hl, R2, bias, svdq::kEpiNone, nullptr, 0, out, out_dtype, ldo,
                                  M, N, K_pad, nullptr, 0, stream, "svdq_linear_gemm");
}

extern "C" size_t svdq_linear_gemm_workspace_bytes(void) { return svdq::workspace_bytes_for(svdq::num_sms() / 2); }

extern "C" int svdq_linear_gemm_ws(const void* a16, const void* w16, const void* mid_hl, const void* up_hl, int R2,
                                   const void* bias, void* out, int out_dtype, int64_t ldo, int M, int N, int K_pad,
                                   void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (workspace && (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return svdq::set_error(SVDQ_ERR_INVALID_ARGUMENT, "svdq_linear_gemm_ws: workspace must be 256-byte aligned");
  if (workspace && workspace_bytes < svdq::workspace_bytes_for(svdq::num_sms() / 2))
    return svdq::set_error(SVDQ_ERR_INVALID_ARGUMENT,
                           "svdq_linear_gemm_ws: workspace smaller than svdq_linear_gemm_workspace_bytes()");
  return svdq::launch_linear_gemm(a16, w16, mid_hl, up_hl, R2, bias, svdq::kEpiNone, nullptr, 0, out, out_dtype, ldo,
                                  M, N, K_pad, workspace, workspace_bytes, stream, "svdq_linear_gemm_ws");
}

extern "C" int svdq_linear_gemm_epi(const void* a16, const void* w16, const void* mid_hl, const void* up_hl, int R2,
                                    const void* bias, int epilogue, const void* aux, int64_t ld_aux, void* out,
                                    int out_dtype, int64_t ldo, int M, int N, int K_pad, void* workspace,
                                    size_t workspace_bytes, cudaStream_t stream) {
  if (workspace && (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return svdq::set_error(SVDQ_ERR_INVALID_ARGUMENT, "svdq_linear_gemm_epi: workspace must be 256-byte aligned");
  if (workspace && workspace_bytes < svdq::workspace_bytes_for(svdq::num_sms() / 2))
    return svdq::set_error(SVDQ_ERR_INVALID_ARGUMENT,
                           "svdq_linear_gemm_epi: workspace smaller than svdq_linear_gemm_workspace_bytes()");
  return svdq::launch_linear_gemm(a16, w16, mid_hl, up_hl, R2, bias, epilogue, aux, ld_aux, out, out_dtype, ldo, M, N,
                                  K_pad, workspace, workspace_bytes, stream, "svdq_linear_gemm_epi");
}

extern "C" int svdq_linear_gemm_group(const svdq_gemm_problem* problems, int num_problems, int R2, int out_dtype,
                                      int M, int K_pad, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (workspace && (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return svdq::set_error(SVDQ_ERR_INVALID_ARGUMENT, "svdq_linear_gemm_group: workspace must be 256-byte aligned");
  if (workspace && workspace_bytes < svdq::workspace_bytes_for(svdq::num_sms() / 2))
    return svdq::set_error(SVDQ_ERR_INVALID_ARGUMENT,
                           "svdq_linear_gemm_group: workspace smaller than svdq_linear_gemm_workspace_bytes()");
  return svdq::launch_linear_gemm_group(problems, num_problems, R2, out_dtype, M, K_pad, workspace, workspace_bytes,
                                        stream, "svdq_linear_gemm_group");
}

extern "C" int svdq_linear_gemm_plan(int tiles, int iters, int max_pairs, int with_workspace, int* out4) {
  if (!out4) return svdq::set_error(SVDQ_ERR_INVALID_ARGUMENT, "svdq_linear_gemm_plan: out4 is NULL");
  if (!(tiles >= 0 && iters > 0 && max_pairs > 0))
    return svdq::set_error(SVDQ_ERR_INVALID_ARGUMENT, "svdq_linear_gemm_plan: bad tiles/iters/max_pairs");
  const svdq::Schedule sc = svdq::plan_schedule(tiles, iters, max_pairs, with_workspace != 0);
  out4[0] = sc.pairs;
  out4[1] = sc.dp_tiles;
  out4[2] = sc.tail_len;
  out4[3] = sc.tail_total;
  return SVDQ_OK;
}

extern "C" int svdq_linear_gemm_schedule(int M, int N, int K_pad, int R2, int with_workspace, int* out4) {
  if (!out4) return svdq::set_error(SVDQ_ERR_INVALID_ARGUMENT, "svdq_linear_gemm_schedule: out4 is NULL");
  if (!(M >= 0 && N > 0 && K_pad > 0 && K_pad % 64 == 0 && R2 >= 0 && R2 % 64 == 0))
    return svdq::set_error(SVDQ_ERR_INVALID_ARGUMENT, "svdq_linear_gemm_schedule: bad M/N/K_pad/R2");
  auto kern = svdq::linear_gemm_kernel<false, svdq::kEpiNone>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)svdq::SMEM_BYTES);
  if (e != cudaSuccess) return svdq::check_cuda(e, "svdq_linear_gemm_schedule: shared memory attribute");
  const int tiles = ((M + 2 * svdq::BM - 1) / (2 * svdq::BM)) * ((N + svdq::BN - 1) / svdq::BN);
  const svdq::Schedule sc = svdq::plan_schedule(tiles, K_pad / 64 + R2 / 64,
                                                svdq::max_resident_pairs(reinterpret_cast<const void*>(kern)),
                                                with_workspace != 0);
  out4[0] = sc.pairs;
  out4[1] = sc.dp_tiles;
  out4[2] = sc.tail_len;
  out4[3] = sc.tail_total;
  return SVDQ_OK;
}

namespace svdq {
namespace {
// The epilogue's activation code on a vector: sigmoid(x) as 1 * sigmoid(x), silu(x) as silu(x) * 1,
// four values per thread as the GEMM epilogue calls it.
template <int EPI>
__global__ void epilogue_act_selftest_kernel(const __nv_bfloat16* in, __nv_bfloat16* out, int n) {
  const int i0 = 4 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (i0 >= n) return;
  __nv_bfloat16 x[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) x[k] = i0 + k < n ? in[i0 + k] : __float2bfloat16_rn(0.0f);
  const __nv_bfloat162 p0 = __halves2bfloat162(x[0], x[1]), p1 = __halves2bfloat162(x[2], x[3]);
  const uint2 xw = make_uint2(*reinterpret_cast<const uint32_t*>(&p0), *reinterpret_cast<const uint32_t*>(&p1));
  const uint2 ones = make_uint2(0x3F803F80u, 0x3F803F80u);  // bf16 1.0 twice
  const uint2 r = EPI == kEpiSigmoidMul
                      ? epi_act4_bf16<EPI>(make_float4(__bfloat162float(x[0]), __bfloat162float(x[1]),
                                                       __bfloat162float(x[2]), __bfloat162float(x[3])), ones)
                      : epi_act4_bf16<EPI>(make_float4(1.0f, 1.0f, 1.0f, 1.0f), xw);
  const __nv_bfloat162 q0 = *reinterpret_cast<const __nv_bfloat162*>(&r.x);
  const __nv_bfloat162 q1 = *reinterpret_cast<const __nv_bfloat162*>(&r.y);
  const __nv_bfloat16 o[4] = {q0.x, q0.y, q1.x, q1.y};
#pragma unroll
  for (int k = 0; k < 4; ++k)
    if (i0 + k < n) out[i0 + k] = o[k];
}
}  // namespace
}  // namespace svdq

extern "C" int svdq_selftest_epilogue_act(int epilogue, const void* in, void* out, int n, cudaStream_t stream) {
  if (!(epilogue == svdq::kEpiSigmoidMul || epilogue == svdq::kEpiSiluMul) || !in || !out || n < 0)
    return svdq::set_error(SVDQ_ERR_INVALID_ARGUMENT, "svdq_selftest_epilogue_act: bad arguments");
  if (n == 0) return SVDQ_OK;
  const dim3 grid((n + 1023) / 1024), block(256);
  const auto* x = static_cast<const __nv_bfloat16*>(in);
  auto* y = static_cast<__nv_bfloat16*>(out);
  if (epilogue == svdq::kEpiSigmoidMul)
    svdq::epilogue_act_selftest_kernel<svdq::kEpiSigmoidMul><<<grid, block, 0, stream>>>(x, y, n);
  else
    svdq::epilogue_act_selftest_kernel<svdq::kEpiSiluMul><<<grid, block, 0, stream>>>(x, y, n);
  return svdq::check_launch("svdq_selftest_epilogue_act");
}
