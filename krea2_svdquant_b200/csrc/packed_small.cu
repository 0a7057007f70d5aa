// Small-batch packed-weight SVDQuant GEMM for sm_100a: integer K-group partial sums in tensor
// memory, rescaled into fp32 accumulators held in registers.
//
//   out[m, n] = sum_g s_w[n, g] * s_a[m, g] * P_g[n, m] + sum_j up_hl[n, j] mid_hl[m, j] + bias[n]
//
//   I8 mode (W4A4, svdq_w4a4_gemm):  P_g = sum_{k in g} q_w[n, k] * q_a[m, k]   tcgen05 kind::i8,
//                                     exact int32; q_a are the activation's int8 codes, s_a its
//                                     per-token group scales.
//   F16 mode (svdq_packed_gemm, M <= 64): P_g = sum_{k in g} q_w[n, k] * a16[m, k]   kind::f16,
//                                     fp32; s_a = 1 (a16 is the W4A16 x_hat, or the W4A4 operand
//                                     q_a * s_a, exact in fp16).
//
// g runs over K ranges inside one weight group and one activation group (the smaller of the two
// group sizes).  This is the W4A4 design of the reference's README formula (README.md:64) with
// the per-group rescale that int MMAs need: the int4 weights go to the tensor core as plain
// integers (int8, or exact small fp16 integers), so a weight costs one integer conversion and
// no scale multiply, and the scale is applied once per group and output element.  The rescale
// costs 2-3 instructions per output element and group, which is cheap while the token count is
// small: the kernel is meant for batches up to 64 tokens per tile, where the weight bytes, not
// the MMAs, bound the layer.  Measured on B200 (tcgen05.mma kind::f16 issue-to-completion, one
// CTA): 44 cycles per instruction for N <= 32, 48 for N = 64, 128 for N = 256, the same with A
// in tensor memory; kind::i8 takes 32 k per instruction where kind::f16 takes 16.
//
// Orientation (swap AB): the CTA's 128 weight rows are the MMA's M (tensor-memory lanes) and the
// tokens its N (TN = 16, 32 or 64).  The weights enter the MMA from tensor memory: converter warps
// turn the packed codes (TMA, 128 rows x 256 k per 16 KiB box, 128-byte swizzle) into int8 or
// fp16 integers in registers and store them with tcgen05.st into a ring of weight stages
// (128 bytes of K per row each: 64 k of fp16 or 128 k of int8).  Token tiles arrive by TMA in the
// same 128-byte-row geometry.  Each K group's MMAs accumulate into their own tensor-memory
// partial buffer; a chunk's buffers form a set, and up to three sets are in flight.  The rescale
// warps (two per lane quarter, thread = weight row, each half of the tokens) load a set, release
// it and fold it into fp32 accumulators.
//
// The low-rank term runs as extra groups at the end of the CTA's K range with scale 1: up_hl
// rows (A, shared memory) times mid_hl tokens (B), kind::f16 with bf16 operands.
//
// Split K: when the tiles would leave SMs idle, a cluster of KS CTAs (KS in {1, 2, 4, 8}) shares
// a tile, each taking a contiguous range of code boxes (the last also takes the low-rank
// groups); after a cluster barrier each CTA adds one slice of rows over all KS partials through
// distributed shared memory, in rank order (deterministic), adds the bias and stores.
//
// Roles (20 warps): warp 0 TMA of code boxes and weight scales; warp 1 tensor-memory allocation
// and the MMA issue; warp 2 TMA of token tiles (and low-rank tiles); warps 4-7 and 16-19 rescale
// and epilogue (two per lane quarter, each half of the tokens); warps 8-15 conversion (two per
// lane quarter, alternate weight stages).  The MMA thread waits by spinning on
// mbarrier.test_wait; every other role polls it with a short nanosleep in between (a suspending
// try_wait costs a few hundred nanoseconds to wake, which this latency-bound pipeline cannot
// hide, and a spinning warp takes issue slots from the MMA thread).  Every wait is bounded (error word
// codes 0x55xx-0x58xx); a wait that runs out raises the CTA's abort flag, every role leaves its
// loop, and all CTAs still meet at the cluster barriers.
#include <algorithm>

#include "svdq_common.cuh"

namespace svdq {
namespace {

constexpr int SB_ROWS = 128;                 // weight rows per CTA (TMEM lanes, MMA M)
constexpr int SB_BOX_K = 256;                // k per code box: 128 bytes of nibbles per row
constexpr uint32_t SB_BOX_BYTES = SB_ROWS * SB_BOX_K / 2;  // 16 KiB
constexpr int SB_PS = 6;                     // code-box ring (shared memory)
constexpr int SB_LS = 2;                     // low-rank A ring
constexpr uint32_t SB_LR_BYTES = SB_ROWS * 64 * 2;  // up_hl tile: 128 rows x 64 bf16
constexpr int SB_CONV_WARPS = 8;
constexpr int SB_RESCALE_WARPS = 8;          // two per lane quarter, each half of the tokens
constexpr int SB_THREADS = 32 * (4 + SB_CONV_WARPS + SB_RESCALE_WARPS);
constexpr uint32_t SB_TMEM_COLS = 512;
constexpr uint32_t SB_STAGE_COLS = 32;       // tensor-memory columns of one weight stage (128 B per row)
constexpr int SB_MAX_SCALES = 8;             // weight scales per row and code box (group 32)
constexpr int SB_MAX_WCH = 4;                // weight chunks in tensor memory, most
constexpr int SB_MAX_TB = 16;                // token chunks in shared memory, most

// Work is synchronized per chunk: 256 k of the K range (one code box), i.e. 4 weight stages of
// fp16 or 2 of int8 and their 16 or 8 MMAs, which accumulate into a set of partial buffers (one
// per K group of the chunk).  One set of waits and commits per chunk keeps the MMA thread's own
// barrier traffic (each mbarrier operation costs it 100-200 cycles) off the MMA critical path.
template <int TN, bool I8>
struct SbLayout {
  static constexpr int kSK = I8 ? 128 : 64;                  // k per weight stage
  static constexpr int kSPB = SB_BOX_K / kSK;                // stages per chunk
  static constexpr uint32_t kPCols = TN < 32 ? 32 : TN;       // columns per partial buffer (32-aligned)
  static constexpr uint32_t kWChunkCols = kSPB * SB_STAGE_COLS;
  static constexpr uint32_t kTokSub = (uint32_t)TN * 128;     // one stage of tokens: TN rows x 128 B
  static constexpr uint32_t kTokChunk = kSPB * kTokSub;
  static constexpr int kTB = (int)(65536 / kTokChunk) < 2 ? 2 : (int)(65536 / kTokChunk) > SB_MAX_TB ? SB_MAX_TB
                                                                                          : (int)(65536 / kTokChunk);
  static constexpr uint32_t kOffP = 0;                                         // code ring
  static constexpr uint32_t kOffB = kOffP + SB_PS * SB_BOX_BYTES;
  static constexpr uint32_t kOffL = kOffB + kTB * kTokChunk;
  static constexpr uint32_t kOffS = kOffL + SB_LS * SB_LR_BYTES;               // weight-scale ring
  static constexpr uint32_t kSBytes = SB_ROWS * SB_MAX_SCALES * 2;
  // I8: activation scales of a chunk (at most 4 groups x TN), staged per rescale warp, double buffered
  static constexpr uint32_t kSaBuf = 4 * TN * 4;
  static constexpr uint32_t kOffA = kOffS + SB_PS * kSBytes;
  static constexpr uint32_t kOffBar = kOffA + (I8 ? SB_RESCALE_WARPS * 2 * kSaBuf : 0);
  static constexpr uint32_t kSmem = kOffBar + 1024 + 1024;                     // barriers + alignment slack
  static_assert(kTokSub % 1024 == 0, "token tiles keep 1 KiB alignment for the 128-byte swizzle");
  static_assert((uint32_t)SB_ROWS * TN * 4 <= kOffB, "split-K partial fits over the code ring");
  static_assert(kSmem <= 227 * 1024, "shared memory per CTA");
};

struct SbBars {
  uint64_t full_p[SB_PS];   // code box and its weight scales landed (TMA bytes)
  uint64_t empty_p[SB_PS];  // code box read (one arrival per converter warp)
  uint64_t empty_s[SB_PS];  // weight scales of the box used (one arrival per rescale warp)
  uint64_t full_b[SB_MAX_TB];   // token chunk (and, for a low-rank chunk, its A) landed
  uint64_t empty_b[SB_MAX_TB];  // MMAs reading the token chunk done (commit)
  uint64_t conv[SB_MAX_WCH];    // weight chunk written to tensor memory (one arrival per converter warp)
  uint64_t empty_a[SB_MAX_WCH]; // MMAs reading the weight chunk done (commit)
  uint64_t empty_l[SB_LS];      // MMAs reading the low-rank A slot done (commit)
  uint64_t pfull[3];            // a chunk's partial set complete (commit)
  uint64_t pempty[3];           // partial set read by the rescale warps (one arrival per rescale warp)
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(SbBars) <= 1024, "barrier block");

struct SbArgs {
  const __half* scales16;   // weight scales, fp16, kernel tile order (svdq_prepare_packed)
  const float* ascales_t;   // I8: activation scales, fp32 [K_pad / a_group][lda_s] (group-major)
  int64_t lda_s;
  const __nv_bfloat16* bias;
  void* out;
  int64_t ldo;
  int M, N, K_pad;
  int w_group, a_group, pg_k;  // weight group, activation group, partial-group width (k)
  int n_lr;                    // low-rank stages (64 columns of R2 each)
  int ks;                      // CTAs per cluster along K
  int units_n;                 // 128-row weight tiles
  int* err;
};

enum : int {
  kSbWaitPackedEmpty = 0x5501,
  kSbWaitTileEmpty = 0x5502,
  kSbWaitLowrankEmpty = 0x5503,
  kSbWaitConvPacked = 0x5601,
  kSbWaitConvEmpty = 0x5602,
  kSbWaitMmaTile = 0x5701,
  kSbWaitMmaConv = 0x5702,
  kSbWaitMmaPartial = 0x5703,
  kSbWaitMmaDrain = 0x5704,
  kSbWaitRescale = 0x5801,
  kSbWaitScales = 0x5802,
};

__device__ __forceinline__ uint32_t h2_sub(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t h2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ float4 lds128f(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ float ldg_f32_volatile(const float* p) {
  float v;
  asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}
// 32 lanes x 8 consecutive 32-bit columns: thread i of the warp gets lane (base + i).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ uint16_t lds16(uint32_t addr) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
__device__ __forceinline__ float ld_dsmem(uint32_t cluster_addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(cluster_addr) : "memory");
  return v;
}
__device__ __forceinline__ void arrive_cta(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// tcgen05.mma kind::i8 (int32 accumulation) with A in tensor memory and B in shared memory.
__device__ __forceinline__ void umma_i8_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// 32 lanes x 32 consecutive 32-bit columns from registers: thread i of the warp writes lane (base + i).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// Instruction descriptors: D fp32 (kind::f16) or s32 (kind::i8), K-major A and B, M = 128.
__host__ __device__ constexpr uint32_t idesc_f16(uint32_t ab_fmt, int n) { return make_idesc(ab_fmt, ab_fmt, SB_ROWS, n); }
__host__ __device__ constexpr uint32_t idesc_i8(int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(SB_ROWS >> 4) << 24);
}

// One 32-bit word of kernel-order codes ([k0 k2 k4 k6 | k1 k3 k5 k7], nibble = q + 8) ->
// F16: four fp16x2 pairs (k0 k1), (k2 k3), (k4 k5), (k6 k7) of the exact integers q;
// I8: two words of int8 q, [k0 k1 k2 k3] and [k4 k5 k6 k7].
__device__ __forceinline__ void codes_to_f16(uint32_t w, uint32_t* o) {
  constexpr uint32_t kExp = 0x64006400u;        // fp16x2 {1024, 1024}
  constexpr uint32_t kOff = 0x64086408u;        // {1032, 1032}: 1024 + the nibble offset 8
  constexpr uint32_t kSixteenth = 0x2C002C00u;  // {1/16, 1/16}
  constexpr uint32_t kNeg72 = 0xD480D480u;      // {-72, -72}: -(1024 + 128) / 16
  const uint32_t w8 = w >> 8;
  o[0] = h2_sub((w & 0x000F000Fu) | kExp, kOff);
  o[1] = h2_fma((w & 0x00F000F0u) | kExp, kSixteenth, kNeg72);  // (1024 + 16 n) / 16 - 72 = n - 8, exact
  o[2] = h2_sub((w8 & 0x000F000Fu) | kExp, kOff);
  o[3] = h2_fma((w8 & 0x00F000F0u) | kExp, kSixteenth, kNeg72);
}
__device__ __forceinline__ void codes_to_i8(uint32_t w, uint32_t* o) {
  const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
  // bytes: lo = [k0 k4 k1 k5], hi = [k2 k6 k3 k7]; n -> n - 8 per byte: (n + 120) ^ 128, no carries
  o[0] = (__byte_perm(lo, hi, 0x6420) + 0x78787878u) ^ 0x80808080u;
  o[1] = (__byte_perm(lo, hi, 0x7531) + 0x78787878u) ^ 0x80808080u;
}

template <int TN, bool I8, bool OUT_F32>
__global__ void __launch_bounds__(SB_THREADS, 1)
    packed_small_kernel(const __grid_constant__ CUtensorMap tm_tok, const __grid_constant__ CUtensorMap tm_codes,
                        const __grid_constant__ CUtensorMap tm_mid, const __grid_constant__ CUtensorMap tm_up,
                        const SbArgs args) {
  using L = SbLayout<TN, I8>;
  constexpr int SK = L::kSK, SPB = L::kSPB, TB = L::kTB;
  constexpr int KSTEP = I8 ? 32 : 16;        // k per MMA
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  SbBars* bars = reinterpret_cast<SbBars*>(gbase + L::kOffBar);
  volatile int* abort_flag = &bars->abort_flag;
  const uint32_t p_ring = base + L::kOffP, b_ring = base + L::kOffB, l_ring = base + L::kOffL,
                 s_ring = base + L::kOffS;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ks = args.ks;
  const int crank = (int)(blockIdx.x % (unsigned)ks);
  const int unit = (int)(blockIdx.x / (unsigned)ks);
  const int units_m = (args.M + TN - 1) / TN;
  // token tiles innermost: the CTAs that share a weight tile run side by side and share its codes in L2
  const int mb = unit % units_m, nb = unit / units_m;
  const int n0 = nb * SB_ROWS, m0 = mb * TN;
  const int n_box = (args.K_pad + SB_BOX_K - 1) / SB_BOX_K;
  const int b0 = (int)((int64_t)crank * n_box / ks), b1 = (int)((int64_t)(crank + 1) * n_box / ks);
  const int k0 = b0 * SB_BOX_K, k1 = min(b1 * SB_BOX_K, args.K_pad);  // this CTA's K range
  const int n_res = (k1 - k0) / SK;                                     // weight stages
  const int n_ch = b1 - b0;                                             // residual chunks
  const int n_lr = crank == ks - 1 ? args.n_lr : 0;                     // low-rank chunks (one stage each)
  const int pg_k = args.pg_k;
  const int lg_steps = __ffs(pg_k / KSTEP) - 1;                         // log2(MMAs per group)
  // group widths are powers of two: shifts, not divisions, on the latency-bound single-warp paths
  const int lg_pg = __ffs(pg_k) - 1, lg_wg = __ffs(args.w_group) - 1, lg_ag = __ffs(args.a_group) - 1;
  const int gpc = SB_BOX_K >> lg_pg;                                    // groups per full chunk
  const int spg = SB_BOX_K >> lg_wg;                                    // weight scales per row and box
  // tensor memory: partial sets, then the weight-chunk ring
  const uint32_t set_cols = (uint32_t)gpc * L::kPCols;
  // as many partial sets (up to 3) as leave room for two weight chunks: the MMAs of chunk c + psets
  // wait for the rescale of chunk c
  const int psets = 3 * set_cols + 2 * L::kWChunkCols <= SB_TMEM_COLS   ? 3
                    : 2 * set_cols + 2 * L::kWChunkCols <= SB_TMEM_COLS ? 2
                                                                        : 1;
  const int wch_fit = (int)((SB_TMEM_COLS - psets * set_cols) / L::kWChunkCols);
  const int WCH = wch_fit > SB_MAX_WCH ? SB_MAX_WCH : wch_fit;
  auto stages_of = [&](int c) { return min(SPB, n_res - c * SPB); };

  auto bar = [&](const uint64_t& b) { return smem_u32(&b); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < SB_PS; ++s) {
      mbar_init(bar(bars->full_p[s]), 1);
      mbar_init(bar(bars->empty_p[s]), SB_CONV_WARPS);
      mbar_init(bar(bars->empty_s[s]), SB_RESCALE_WARPS);
    }
    for (int s = 0; s < TB; ++s) {
      mbar_init(bar(bars->full_b[s]), 1);
      mbar_init(bar(bars->empty_b[s]), 1);
    }
    for (int s = 0; s < SB_MAX_WCH; ++s) {
      mbar_init(bar(bars->conv[s]), SB_CONV_WARPS);
      mbar_init(bar(bars->empty_a[s]), 1);
    }
    for (int s = 0; s < SB_LS; ++s) mbar_init(bar(bars->empty_l[s]), 1);
    for (int s = 0; s < 3; ++s) {
      mbar_init(bar(bars->pfull[s]), 1);
      mbar_init(bar(bars->pempty[s]), SB_RESCALE_WARPS);
    }
    mbar_init(bar(bars->mma_done), 1);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tma_desc(&tm_tok);
    prefetch_tma_desc(&tm_codes);
    if (args.n_lr > 0) {
      prefetch_tma_desc(&tm_mid);
      prefetch_tma_desc(&tm_up);
    }
  }
  if (warp == 1) {
    tmem_alloc_1(smem_u32(&bars->tmem_base), SB_TMEM_COLS);
    tmem_relinquish_1();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const uint32_t tmem_w = tmem + psets * set_cols;  // weight chunks after the partial sets
  pdl_wait();  // operands may come from the previous kernel on the stream
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ code boxes + their weight scales
      uint32_t filled = 0, par = 0;
      bool ok = true;
      const uint32_t sbytes = (uint32_t)(SB_ROWS * spg * 2);
      for (int it = 0; it < n_ch && ok; ++it) {
        const int s = it % SB_PS;
        const uint32_t ph = (uint32_t)(it / SB_PS) & 1u;
        if (!(ok = wait_spin(bar(bars->empty_p[s]), ph ^ 1u, abort_flag, args.err, kSbWaitPackedEmpty))) break;
        if (!(ok = wait_spin(bar(bars->empty_s[s]), ph ^ 1u, abort_flag, args.err, kSbWaitPackedEmpty))) break;
        mbar_arrive_expect_tx(bar(bars->full_p[s]), SB_BOX_BYTES + sbytes);
        tma_load_2d(p_ring + (uint32_t)s * SB_BOX_BYTES, &tm_codes, bar(bars->full_p[s]), (b0 + it) * (SB_BOX_K / 2), n0);
        bulk_g2s(s_ring + (uint32_t)s * L::kSBytes, args.scales16 + ((int64_t)nb * n_box + b0 + it) * SB_ROWS * spg,
                 sbytes, bar(bars->full_p[s]));
        filled |= 1u << s;
        par = (par & ~(1u << s)) | (ph << s);
      }
      if (!ok)
        for (int s = 0; s < SB_PS; ++s)
          if (filled & (1u << s)) mbar_wait_drain(bar(bars->full_p[s]), (par >> s) & 1u, 100000000ull);
    }
  } else if (warp == 2) {
    if (lane == 0) {
      // ------------------------------------------------ token chunks (+ low-rank A)
      uint32_t filled = 0, par = 0;
      bool ok = true;
      for (int it = 0; it < n_ch + n_lr && ok; ++it) {
        const int s = it % TB;
        const uint32_t ph = (uint32_t)(it / TB) & 1u;
        if (!(ok = wait_spin(bar(bars->empty_b[s]), ph ^ 1u, abort_flag, args.err, kSbWaitTileEmpty))) break;
        const uint32_t fb = bar(bars->full_b[s]);
        const uint32_t bdst = b_ring + (uint32_t)s * L::kTokChunk;
        if (it < n_ch) {
          const int st = stages_of(it);
          mbar_arrive_expect_tx(fb, (uint32_t)st * L::kTokSub);
          for (int j = 0; j < st; ++j)
            tma_load_2d(bdst + (uint32_t)j * L::kTokSub, &tm_tok, fb, k0 + (it * SPB + j) * SK, m0);
        } else {
          const int j = it - n_ch, ls = j % SB_LS;
          const uint32_t lph = (uint32_t)(j / SB_LS) & 1u;
          if (!(ok = wait_spin(bar(bars->empty_l[ls]), lph ^ 1u, abort_flag, args.err, kSbWaitLowrankEmpty)))
            break;
          mbar_arrive_expect_tx(fb, L::kTokSub + SB_LR_BYTES);
          tma_load_2d(l_ring + (uint32_t)ls * SB_LR_BYTES, &tm_up, fb, j * 64, n0);
          tma_load_2d(bdst, &tm_mid, fb, j * 64, m0);
        }
        filled |= 1u << s;
        par = (par & ~(1u << s)) | (ph << s);
      }
      if (!ok)
        for (int s = 0; s < TB; ++s)
          if (filled & (1u << s)) mbar_wait_drain(bar(bars->full_b[s]), (par >> s) & 1u, 100000000ull);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issue, one chunk per round of waits
      const uint32_t idesc_res = I8 ? idesc_i8(TN) : idesc_f16(0u /*f16*/, TN);
      const uint32_t idesc_lr = idesc_f16(kFmtBF16, TN);
      bool ok = true;
      int tb = 0, wc = 0, ps = 0;
      uint32_t tph = 0, wph = 0, pph = 0;
      const int step_mask = (1 << lg_steps) - 1;
      for (int c = 0; c < n_ch + n_lr && ok; ++c) {
        const bool res = c < n_ch;
        if (!(ok = mbar_spin_wait(bar(bars->full_b[tb]), tph, abort_flag, args.err, kSbWaitMmaTile))) break;
        if (res && !(ok = mbar_spin_wait(bar(bars->conv[wc]), wph, abort_flag, args.err, kSbWaitMmaConv))) break;
        if (!(ok = mbar_spin_wait(bar(bars->pempty[ps]), pph ^ 1u, abort_flag, args.err, kSbWaitMmaPartial))) break;
        tc_fence_after();
        const uint32_t dset = tmem + (uint32_t)ps * set_cols;
        const uint32_t tok = b_ring + (uint32_t)tb * L::kTokChunk;
        if (res) {
          const int st = stages_of(c);
          const uint32_t wbase = tmem_w + (uint32_t)wc * L::kWChunkCols;
          for (int j = 0; j < st; ++j) {
            const uint64_t db = desc_k_sw128(tok + (uint32_t)j * L::kTokSub);
            const uint32_t ta = wbase + (uint32_t)j * SB_STAGE_COLS;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const int step = j * 4 + kk;
              const uint32_t d = dset + (uint32_t)(step >> lg_steps) * L::kPCols;
              const uint32_t acc = (step & step_mask) ? 1u : 0u;
              if constexpr (I8) umma_i8_tmem_a(d, ta + 8u * kk, db + (uint64_t)(2 * kk), idesc_res, acc);
              else umma_f16_1_tmem_a(d, ta + 8u * kk, db + (uint64_t)(2 * kk), idesc_res, acc);
            }
          }
          umma_commit_1(bar(bars->pfull[ps]));
          umma_commit_1(bar(bars->empty_a[wc]));
          if (++wc == WCH) { wc = 0; wph ^= 1u; }
        } else {
          const int ls = (c - n_ch) % SB_LS;
          const uint64_t db = desc_k_sw128(tok);
          const uint64_t da = desc_k_sw128(l_ring + (uint32_t)ls * SB_LR_BYTES);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16_1(dset, da + (uint64_t)(2 * kk), db + (uint64_t)(2 * kk), idesc_lr, kk > 0 ? 1u : 0u);
          umma_commit_1(bar(bars->pfull[ps]));
          umma_commit_1(bar(bars->empty_l[ls]));
        }
        umma_commit_1(bar(bars->empty_b[tb]));
        if (++tb == TB) { tb = 0; tph ^= 1u; }
        if (++ps == psets) { ps = 0; pph ^= 1u; }
      }
      // no MMA may be in flight when the CTA frees tensor memory or exits
      umma_commit_1(bar(bars->mma_done));
      if (!mbar_wait_drain(bar(bars->mma_done), 0, 1000000000ull)) {
        *abort_flag = 1;
        atomicCAS(args.err, 0, kSbWaitMmaDrain);
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp >= 8 && warp < 16) {
    // ------------------------------------------------ conversion: codes -> integers in tensor memory
    // Two warps per lane quarter split each chunk's stages (alternately); a thread converts its
    // row's 128 bytes of operand per stage and stores them with one tcgen05.st.  Each warp
    // arrives once per chunk on the chunk's barriers, stages or not.
    const int q = warp & 3, half = (warp - 8) >> 2;
    const int row = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const uint32_t r7 = (uint32_t)(row & 7);
    constexpr int kChunks16 = SK / 32;  // 16-byte code chunks per stage and row
    constexpr int kMine = SPB / 2;      // stages per chunk of this warp (a full chunk)
    bool ok = true;
    int wc = 0;
    uint32_t wph = 0;
    for (int c = 0; c < n_ch && ok; ++c) {
      const int ps = c % SB_PS, st = stages_of(c);
      if (!(ok = __all_sync(0xffffffffu, wait_spin(bar(bars->full_p[ps]), (uint32_t)(c / SB_PS) & 1u, abort_flag,
                                                   args.err, kSbWaitConvPacked))))
        break;
      uint32_t w[kMine][4 * kChunks16];
      const uint32_t rbase = p_ring + (uint32_t)ps * SB_BOX_BYTES + (uint32_t)row * 128u;
#pragma unroll
      for (int i = 0; i < kMine; ++i) {
        const int j = half + 2 * i;  // stage within the chunk
#pragma unroll
        for (int cc = 0; cc < kChunks16; ++cc) {
          const uint4 v = j < st ? lds128(rbase + ((((uint32_t)(j * kChunks16 + cc)) ^ r7) << 4)) : make_uint4(0, 0, 0, 0);
          w[i][4 * cc] = v.x;
          w[i][4 * cc + 1] = v.y;
          w[i][4 * cc + 2] = v.z;
          w[i][4 * cc + 3] = v.w;
        }
      }
      __syncwarp();
      if (lane == 0) arrive_cta(bar(bars->empty_p[ps]));  // every lane has read its codes
      if (!(ok = __all_sync(0xffffffffu, wait_spin(bar(bars->empty_a[wc]), wph ^ 1u, abort_flag, args.err,
                                                   kSbWaitConvEmpty))))
        break;
      tc_fence_after();
#pragma unroll
      for (int i = 0; i < kMine; ++i) {
        const int j = half + 2 * i;
        if (j < st) {
          uint32_t o[32];
#pragma unroll
          for (int e = 0; e < 4 * kChunks16; ++e) {
            if constexpr (I8) codes_to_i8(w[i][e], o + 2 * e);
            else codes_to_f16(w[i][e], o + 4 * e);
          }
          tmem_st32(tmem_w + lane_off + (uint32_t)wc * L::kWChunkCols + (uint32_t)j * SB_STAGE_COLS, o);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) arrive_cta(bar(bars->conv[wc]));
      if (++wc == WCH) { wc = 0; wph ^= 1u; }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------ rescale: partials -> fp32 accumulators
    // warps 4-7 take tokens [0, TN/2) and warps 16-19 tokens [TN/2, TN) of the same rows
    const int q = warp & 3, rh = warp >= 16 ? 1 : 0;
    constexpr int TH = TN / 2;
    const int row = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    float acc[TH];
#pragma unroll
    for (int t = 0; t < TH; ++t) acc[t] = 0.f;
    bool ok = true;
    // I8: a chunk's activation scales ([group][token], fp32) are loaded from global memory one chunk
    // ahead into registers, then staged in this warp's shared-memory buffer (reads broadcast)
    constexpr int kSaRegs = I8 ? (4 * TN + 31) / 32 : 1;
    float sa_pre[kSaRegs];
    const int rw = q + 4 * rh;  // rescale warp index
    const uint32_t sa_smem = base + L::kOffA + (uint32_t)rw * 2u * L::kSaBuf;
    float* sa_gen = reinterpret_cast<float*>(gbase + L::kOffA + (uint32_t)rw * 2u * L::kSaBuf);
    auto sa_fetch = [&](int c) {  // chunk c's scales -> sa_pre (every lane its elements)
      if constexpr (I8) {
        if (c < n_ch) {
          const int ngc = (stages_of(c) * SK) >> lg_pg, pg0 = c * gpc;
#pragma unroll
          for (int j = 0; j < kSaRegs; ++j) {
            const int e = lane + 32 * j, g = e / TN, t = e % TN;
            // volatile: issued here, a chunk before its use, not sunk next to the use
            sa_pre[j] = g < ngc ? ldg_f32_volatile(args.ascales_t + (int64_t)((k0 + ((pg0 + g) << lg_pg)) >> lg_ag) *
                                                                        args.lda_s + m0 + t)
                                : 0.f;
          }
        }
      }
    };
    auto sa_stage = [&](int c) {  // sa_pre -> buffer (c & 1)
      if constexpr (I8) {
        __syncwarp();
#pragma unroll
        for (int j = 0; j < kSaRegs; ++j) {
          const int e = lane + 32 * j;
          if (e < 4 * TN) sa_gen[(c & 1) * 4 * TN + e] = sa_pre[j];
        }
        __syncwarp();
      }
    };
    sa_fetch(0);
    sa_stage(0);
    // partial buffers loaded per batch of groups (about 64 registers), one tcgen05.wait::ld each
    constexpr int GB = TH <= 8 ? 4 : TH <= 16 ? 2 : 1;
    int ps = 0;
    uint32_t pph = 0;
    for (int c = 0; c < n_ch + n_lr && ok; ++c) {
      const bool res = c < n_ch;
      const int bps = c % SB_PS;
      sa_fetch(c + 1);
      if (res) ok = wait_spin(bar(bars->full_p[bps]), (uint32_t)(c / SB_PS) & 1u, abort_flag, args.err, kSbWaitScales);
      ok = ok && wait_spin(bar(bars->pfull[ps]), pph, abort_flag, args.err, kSbWaitRescale);
      if (!(ok = __all_sync(0xffffffffu, ok))) break;
      tc_fence_after();
      const int ng = res ? (stages_of(c) * SK) >> lg_pg : 1;
      const uint32_t sset = tmem + lane_off + (uint32_t)ps * set_cols;
      constexpr int CW = TH;  // this warp's columns: 8, 16 or 32
      for (int g0 = 0; g0 < ng; g0 += GB) {
#pragma unroll
        for (int h = 0; h < 1; ++h) {
          uint32_t v[GB][CW];
#pragma unroll
          for (int b = 0; b < GB; ++b) {
            if (g0 + b < ng) {
              const uint32_t src = sset + (uint32_t)(g0 + b) * L::kPCols + (uint32_t)(rh * TH);
              if constexpr (CW == 8) tmem_ld8(src, reinterpret_cast<uint32_t(&)[8]>(v[b][0]));
              else if constexpr (CW == 16) tmem_ld16(src, reinterpret_cast<uint32_t(&)[16]>(v[b][0]));
              else tmem_ld32(src, reinterpret_cast<uint32_t(&)[32]>(v[b][0]));
            }
          }
          tmem_ld_wait();
#pragma unroll
          for (int b = 0; b < GB; ++b)
#pragma unroll
            for (int t = 0; t < CW; ++t) asm volatile("" : "+r"(v[b][t]));  // no use before the wait
          if (g0 + GB >= ng) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) arrive_cta(bar(bars->pempty[ps]));  // the MMA may refill the set
          }
          float* a = acc;
#pragma unroll
          for (int b = 0; b < GB; ++b) {
            const int g = g0 + b;
            if (g >= ng) break;
            if (!res) {
#pragma unroll
              for (int t = 0; t < CW; ++t) a[t] += __uint_as_float(v[b][t]);
              continue;
            }
            const float sw = __half2float(__ushort_as_half(
                lds16(s_ring + (uint32_t)bps * L::kSBytes + 2u * (uint32_t)(row * spg + ((g << lg_pg) >> lg_wg)))));
            if constexpr (I8) {
              const uint32_t sa_row = sa_smem + (uint32_t)(((c & 1) * 4 + g) * TN + rh * TH) * 4u;
#pragma unroll
              for (int t = 0; t < CW; t += 4) {
                const float4 s4 = lds128f(sa_row + 4u * t);
                a[t] = fmaf((float)(int)v[b][t], sw * s4.x, a[t]);
                a[t + 1] = fmaf((float)(int)v[b][t + 1], sw * s4.y, a[t + 1]);
                a[t + 2] = fmaf((float)(int)v[b][t + 2], sw * s4.z, a[t + 2]);
                a[t + 3] = fmaf((float)(int)v[b][t + 3], sw * s4.w, a[t + 3]);
              }
            } else {
#pragma unroll
              for (int t = 0; t < CW; ++t) a[t] = fmaf(__uint_as_float(v[b][t]), sw, a[t]);
            }
          }
        }
      }
      if (res) {
        __syncwarp();
        if (lane == 0) arrive_cta(bar(bars->empty_s[bps]));  // done with the box's weight scales
      }
      sa_stage(c + 1);
      if (++ps == psets) { ps = 0; pph ^= 1u; }
    }
    // ---------------------------------------------- epilogue: out, or this CTA's split-K partial
    // (every MMA has completed once the last partial was read: the partial may reuse the code ring)
    if (ok && !*abort_flag) {
      const int n = n0 + row;
      if (ks > 1) {
        float* part = reinterpret_cast<float*>(gbase);  // [TN][128]
#pragma unroll
        for (int t = 0; t < TH; ++t) part[(rh * TH + t) * SB_ROWS + row] = acc[t];
      } else if (n < args.N) {
        const float b = args.bias ? __bfloat162float(args.bias[n]) : 0.f;
#pragma unroll
        for (int t = 0; t < TH; ++t) {
          const int m = m0 + rh * TH + t;
          if (m < args.M) {
            const float y = acc[t] + b;
            if constexpr (OUT_F32) static_cast<float*>(args.out)[(int64_t)m * args.ldo + n] = y;
            else static_cast<__nv_bfloat16*>(args.out)[(int64_t)m * args.ldo + n] = __float2bfloat16_rn(y);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (ks > 1) {
    // ------------------------------------------------ split-K: sum the cluster's partials
    cluster_sync();  // every CTA's partial is in its shared memory
    const int rows = SB_ROWS / ks;
    for (int o = threadIdx.x; o < rows * TN; o += SB_THREADS) {
      const int rl = o % rows, col = o / rows;
      const int row = crank * rows + rl;
      const int n = n0 + row, m = m0 + col;
      const uint32_t off = (uint32_t)(col * SB_ROWS + row) * 4u;
      float pv[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) pv[c] = c < ks ? ld_dsmem(mapa_shared(base + off, (uint32_t)c)) : 0.f;
      float y = 0.f;
#pragma unroll
      for (int c = 0; c < 8; ++c) y += pv[c];  // rank order
      if (n < args.N && m < args.M && !*abort_flag) {
        if (args.bias) y += __bfloat162float(args.bias[n]);
        if constexpr (OUT_F32) static_cast<float*>(args.out)[(int64_t)m * args.ldo + n] = y;
        else static_cast<__nv_bfloat16*>(args.out)[(int64_t)m * args.ldo + n] = __float2bfloat16_rn(y);
      }
    }
    cluster_sync();  // no CTA leaves while another still reads its shared memory
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_1(tmem, SB_TMEM_COLS);
  }
}

struct SbPlan {
  int tn, ks, units_n, units_m;
};

int sb_pick_tn(int M, int pg_k) { return M <= 16 ? 16 : (M <= 32 || pg_k < 64) ? 32 : 64; }

// Split factor: among KS in {1, 2, 4, 8} (at least two code boxes per CTA), the fewest waves of
// CTAs (one per SM), then the fullest last wave; ties go to the smaller KS.
SbPlan sb_plan(int M, int N, int K_pad, int pg_k) {
  SbPlan p;
  p.tn = sb_pick_tn(M, pg_k);
  p.units_n = (N + SB_ROWS - 1) / SB_ROWS;
  p.units_m = (M + p.tn - 1) / p.tn;
  const int n_box = (K_pad + SB_BOX_K - 1) / SB_BOX_K;
  const long long units = (long long)p.units_n * p.units_m;
  const long long slots = num_sms();
  p.ks = 1;
  double best = -1.0;
  long long best_waves = 1ll << 40;
  for (int ks = 1; ks <= 8 && (ks == 1 || n_box / ks >= 2); ks *= 2) {
    const long long ctas = units * ks;
    const long long waves = (ctas + slots - 1) / slots;
    const double fill = (double)ctas / (double)(waves * slots);
    if (waves < best_waves || (waves == best_waves && fill > best + 1e-9)) {
      best_waves = waves;
      best = fill;
      p.ks = ks;
    }
  }
  return p;
}

template <int TN, bool I8, bool OUT_F32>
int launch_sb(const CUtensorMap& tt, const CUtensorMap& tc, const CUtensorMap& tmid, const CUtensorMap& tup,
              const SbArgs& a, int grid, cudaStream_t stream) {
  auto kern = packed_small_kernel<TN, I8, OUT_F32>;
  constexpr uint32_t smem = SbLayout<TN, I8>::kSmem;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return check_cuda(e, "packed small-batch GEMM: shared memory attribute");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(SB_THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = a.ks;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, kern, tt, tc, tmid, tup, a);
  if (e != cudaSuccess) return check_cuda(e, "packed small-batch GEMM launch");
  return check_launch("packed small-batch GEMM launch");
}

template <bool I8, bool OUT_F32>
int launch_sb_tn(int tn, const CUtensorMap& tt, const CUtensorMap& tc, const CUtensorMap& tmid,
                 const CUtensorMap& tup, const SbArgs& a, int grid, cudaStream_t stream) {
  switch (tn) {
    case 16: return launch_sb<16, I8, OUT_F32>(tt, tc, tmid, tup, a, grid, stream);
    case 32: return launch_sb<32, I8, OUT_F32>(tt, tc, tmid, tup, a, grid, stream);
    default: return launch_sb<64, I8, OUT_F32>(tt, tc, tmid, tup, a, grid, stream);
  }
}

}  // namespace

// Shared by svdq_w4a4_gemm (int8 activation codes) and svdq_packed_gemm's small-batch path (fp16
// activation operand).  Argument checks are the callers'.
int packed_small_gemm(const void* act, bool i8, const float* ascales_t, int64_t lda_s, int a_group, const void* codes,
                      const void* scales16, int w_group, const void* mid_hl, const void* up_hl, int R2,
                      const void* bias, void* out, int out_dtype, int64_t ldo, int M, int N, int K_pad,
                      cudaStream_t stream) {
  int* err = device_error_word();
  if (!err) return set_error(SVDQ_ERR_CUDA, "packed small-batch GEMM: device error word unavailable");
  const int pg_k = std::min(w_group, i8 ? a_group : w_group);
  const SbPlan p = sb_plan(M, N, K_pad, pg_k);
  CUtensorMap tt, tc, tmid, tup;
  int st;
  if ((st = make_tma_2d(&tt, i8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, act, K_pad, M,
                        (uint64_t)K_pad * (i8 ? 1 : 2), i8 ? 128 : 64, p.tn, CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if ((st = make_tma_2d(&tc, CU_TENSOR_MAP_DATA_TYPE_UINT8, codes, K_pad / 2, N, (uint64_t)K_pad / 2, SB_BOX_K / 2,
                        SB_ROWS, CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if (R2 > 0) {
    if ((st = make_tma_2d(&tmid, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, mid_hl, R2, M, (uint64_t)R2 * 2, 64, p.tn,
                          CU_TENSOR_MAP_SWIZZLE_128B)))
      return st;
    if ((st = make_tma_2d(&tup, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, up_hl, R2, N, (uint64_t)R2 * 2, 64, SB_ROWS,
                          CU_TENSOR_MAP_SWIZZLE_128B)))
      return st;
  } else {
    tmid = tt;
    tup = tt;
  }
  SbArgs a;
  a.scales16 = static_cast<const __half*>(scales16);
  a.ascales_t = ascales_t;
  a.lda_s = lda_s;
  a.bias = static_cast<const __nv_bfloat16*>(bias);
  a.out = out;
  a.ldo = ldo;
  a.M = M;
  a.N = N;
  a.K_pad = K_pad;
  a.w_group = w_group;
  a.a_group = i8 ? a_group : w_group;
  a.pg_k = pg_k;
  a.n_lr = R2 / 64;
  a.ks = p.ks;
  a.units_n = p.units_n;
  a.err = err;
  const int grid = p.units_n * p.units_m * p.ks;
  const bool f32 = out_dtype == SVDQ_FP32;
  if (i8) return f32 ? launch_sb_tn<true, true>(p.tn, tt, tc, tmid, tup, a, grid, stream)
                     : launch_sb_tn<true, false>(p.tn, tt, tc, tmid, tup, a, grid, stream);
  return f32 ? launch_sb_tn<false, true>(p.tn, tt, tc, tmid, tup, a, grid, stream)
             : launch_sb_tn<false, false>(p.tn, tt, tc, tmid, tup, a, grid, stream);
}

int packed_small_plan(int M, int N, int K_pad, int* out4) {
  const SbPlan p = sb_plan(M, N, K_pad, 64);
  out4[0] = p.tn;
  out4[1] = p.ks;
  out4[2] = p.units_n * p.units_m * p.ks;
  out4[3] = 1;
  return SVDQ_OK;
}

}  // namespace svdq

extern "C" int svdq_w4a4_gemm(const void* codes8, const float* ascales_t, int64_t lda_s, int a_group,
                              const void* codes, const void* scales16, int w_group, const void* mid_hl,
                              const void* up_hl, int R2, const void* bias, void* out, int out_dtype, int64_t ldo,
                              int M, int N, int K_pad, cudaStream_t stream) {
  using namespace svdq;
  SVDQ_REQUIRE(codes8 && ascales_t && codes && scales16 && out, "svdq_w4a4_gemm: null operand pointer");
  SVDQ_REQUIRE(M >= 0 && N > 0 && K_pad > 0 && K_pad % 128 == 0,
               "svdq_w4a4_gemm: K_pad must be a positive multiple of 128");
  SVDQ_REQUIRE((w_group == 64 || w_group == 128 || w_group == 256) && K_pad % w_group == 0,
               "svdq_w4a4_gemm: w_group must be 64, 128 or 256 and divide K_pad");
  SVDQ_REQUIRE((a_group == 64 || a_group == 128) && K_pad % a_group == 0,
               "svdq_w4a4_gemm: a_group must be 64 or 128 and divide K_pad");
  SVDQ_REQUIRE(lda_s >= ((int64_t)M + 63) / 64 * 64 && lda_s % 4 == 0,
               "svdq_w4a4_gemm: lda_s must be a multiple of 4 and >= M rounded up to 64");
  SVDQ_REQUIRE((reinterpret_cast<uintptr_t>(codes8) & 15u) == 0 && (reinterpret_cast<uintptr_t>(ascales_t) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(scales16) & 15u) == 0 && (reinterpret_cast<uintptr_t>(codes) & 15u) == 0,
               "svdq_w4a4_gemm: codes8, ascales_t, codes and scales16 must be 16-byte aligned");
  SVDQ_REQUIRE(N % 8 == 0 && ldo >= N && ldo % 8 == 0, "svdq_w4a4_gemm: N and ldo must be multiples of 8, ldo >= N");
  SVDQ_REQUIRE(R2 >= 0 && R2 % 64 == 0, "svdq_w4a4_gemm: R2 must be a multiple of 64");
  SVDQ_REQUIRE(R2 == 0 || (mid_hl && up_hl), "svdq_w4a4_gemm: mid_hl/up_hl are NULL");
  SVDQ_REQUIRE(out_dtype == SVDQ_BF16 || out_dtype == SVDQ_FP32, "svdq_w4a4_gemm: out_dtype must be bf16 or fp32");
  SVDQ_REQUIRE(!bias || (reinterpret_cast<uintptr_t>(bias) & 1u) == 0, "svdq_w4a4_gemm: bias must be 2-byte aligned");
  if (M == 0) return SVDQ_OK;
  return packed_small_gemm(codes8, true, ascales_t, lda_s, a_group, codes, scales16, w_group, mid_hl, up_hl, R2, bias,
                           out, out_dtype, ldo, M, N, K_pad, stream);
}
