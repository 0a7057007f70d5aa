// Packed-weight SVDQuant linear GEMM for sm_100a (tcgen05 + TMA + TMEM).
//
//   out[m, n] = sum_k a16[m,k] * (q_w[n,k] * s_w[n, k/G]) + sum_j mid_hl[m,j] up_hl[n,j] + bias[n]
//
// The INT4 weight stays packed in HBM (half a byte per weight, the checkpoint's size): each CTA
// streams its rows' codes with TMA, converts them to fp16 in registers and stores them into tensor
// memory, where the tensor core reads its A operand.  No fp16 copy of the weight exists, so a layer
// costs its packed bytes in memory, and a small batch reads 4x fewer weight bytes than a kernel
// over a dequantized weight.
//
// Orientation (swap AB): the weight rows are the MMA's M (128 TMEM lanes per CTA) and the tokens
// its N (TN columns, 16 to 256), so 16 tokens cost a 128x16 MMA instead of most of a 128x256 tile,
// and up to 256 tokens share one conversion of each weight tile.
// The accumulator lands in TMEM as [weight row][token] and leaves transposed.
//
// Tensor memory holds the accumulator (columns [0, TN)) and a ring of converted weight stages
// (32 columns = 64 fp16 of K per row each): 12 to 15 stages deep, so the conversion runs well
// ahead of the MMAs and no stage waits for a full convert -> MMA -> release round trip.  A
// converter thread owns one weight row (its TMEM lane) and a quarter of a stage's K; tcgen05.st moves
// its 16 fp16 values straight from registers to its lane, so the weights never touch shared memory.
//
// Conversion.  The load-time preparation (svdq_prepare_packed) reorders the nibbles of each 32-bit
// word to [k0 k2 k4 k6 | k1 k3 k5 k7] (low half-word holds the even k), so one AND/OR per pair puts
// two codes into the mantissas of an fp16x2 pair with exponent 2^10: 1024 + n (even pair) or
// 1024 + 16 n (odd pair, whose nibbles sit 4 bits higher).  One subtraction gives the exact code
// (n - 8 or 16 (n - 8)), one multiplication the exact product with the group scale (s or s / 16):
// q * s has at most 3 + 8 significant bits for a bf16-valued scale, so it is exact in fp16, and
// equals the load-time fp16 operand of the other GEMM bit for bit.  13 instructions per 8 weights.
//
// Low-rank stages (mid_hl x up_hl, bf16) take their A operand from shared memory (TMA), as the
// other GEMM does.
//
// Split K.  When the tiles would leave SMs idle, a cluster of KS CTAs (KS in {1, 2, 4, 8}) shares a
// tile, each taking one contiguous K range; the last one also takes the low-rank stages.  Each
// CTA parks its fp32 partial in its own shared memory, and after a cluster barrier each CTA sums
// one slice of rows over all KS partials through distributed shared memory, in rank order (a
// fixed order: results are deterministic), adds the bias and stores.
//
// The converters convert a group into registers while the MMAs still hold its TMEM slots, store it
// once they are free and publish it right away (tcgen05.wait::st, then the group's barrier).
// Publishing only after converting the next group (to hide the store drain) put a conversion on
// the MMAs' critical path: measured at 256 tokens, the MMA thread then idled 0.3-0.5 us per group.
//
// Roles (20 warps): warp 0 TMA of packed codes (4-deep ring of 128 rows x 256 k groups, 128-byte
// swizzle so the converters' shared loads are free of bank conflicts); warp 2 TMA of
// the token tiles (a16, or mid_hl with up_hl for the low-rank stages); warp 1 TMEM allocation and
// the MMA issue; warps 4-19 conversion (four warps per TMEM lane quarter); warps 4-7 the epilogue.
// The single-thread roles (TMA producers, MMA issue) wait by spinning on mbarrier.test_wait; the 16
// converter warps and the epilogue poll test_wait with a short nanosleep in between, so that waiting
// converters take few issue slots from the MMA thread on their SMSP (a suspending try_wait takes
// 0.13-0.36 us to return even on a completed phase, twice per code group on the converters' chain).
// The converters publish a code group's four TMEM stages as soon as they are stored, and the MMAs
// release them, with one barrier per group.
// Every wait is bounded (error word codes 0x51xx-0x54xx); a wait that runs out raises the CTA's
// abort flag and every role leaves its loop, so all CTAs still meet at the cluster barriers.
#include <algorithm>

#include "svdq_common.cuh"

namespace svdq {
namespace {

constexpr int PW_ROWS = 128;                          // weight rows per CTA (TMEM lanes)
constexpr int PW_KB = 64;                             // k per stage
constexpr int PW_SUB = 4;                             // 64-k stages per code group (one TMA box)
constexpr int PW_PSTAGES = 4;                         // code-group ring (shared memory)
constexpr int PW_LSTAGES = 2;                         // low-rank A ring (shared memory)
constexpr uint32_t PW_P_BYTES = PW_ROWS * PW_SUB * PW_KB / 2;  // 16 KiB of codes: 128 rows x 128 bytes
constexpr int PW_GROUP_K = PW_SUB * PW_KB;                      // 256 k per code group
constexpr uint32_t PW_S_BYTES = PW_ROWS * (PW_GROUP_K / 32) * 2;  // group scales of a code group (G >= 32)
constexpr uint32_t PW_A_BYTES = PW_ROWS * PW_KB * 2;  // 16 KiB: a low-rank A stage
constexpr int PW_CONV_WARPS = 16;
constexpr int PW_THREADS = 32 * (4 + PW_CONV_WARPS);
constexpr uint32_t PW_TMEM_COLS = 512;
constexpr uint32_t PW_STAGE_COLS = PW_KB / 2;         // TMEM columns of one converted stage
static_assert(PW_CONV_WARPS * 32 * 8 * PW_SUB == (int)PW_P_BYTES, "four 8-byte pieces of codes per converter thread");

// W16: the weight arrives as fp16 tiles (the load-time q * s operand) by TMA into a shared-memory
// ring and the MMA reads A from there; no conversion.  Otherwise packed codes are converted into a
// TMEM ring.
template <int TN, bool W16 = false>
struct PwLayout {
  static constexpr uint32_t kAccCols = TN < 32 ? 32 : TN;                     // accumulator columns
  static constexpr int kAStages = std::min<int>(12, (PW_TMEM_COLS - kAccCols) / PW_STAGE_COLS) / PW_SUB * PW_SUB;
  static constexpr uint32_t kB = (uint32_t)TN * PW_KB * 2;                    // token tile bytes per stage
  // W16 with up to 64 tokens: two CTAs per SM (8 warps, the accumulator's TMEM columns only, about
  // 106 KB of shared memory), so each SM streams the weight through two TMA rings
  static constexpr bool kTwoPerSm = W16 && TN <= 64;
  static constexpr int kBStages = kTwoPerSm ? (kB <= 2048 ? 8 : kB <= 4096 ? 4 : 3)
                                            : kB <= 2048 ? 16 : kB <= 4096 ? 12 : kB <= 16384 ? 6 : 3;
  static constexpr uint32_t kOffL = 0;                                        // low-rank A ring
  static constexpr uint32_t kOffB = kOffL + PW_LSTAGES * PW_A_BYTES;
  static constexpr uint32_t kOffP = kOffB + kBStages * kB;
  static constexpr int kWStages = !W16 ? 0 : kTwoPerSm ? 3 : 6;             // fp16 weight ring (W16)
  static constexpr int kThreads = kTwoPerSm ? 256 : PW_THREADS;             // W16: no converter warps
  static constexpr uint32_t kTmemCols = !W16 ? PW_TMEM_COLS : kAccCols <= 32 ? 32 : kAccCols <= 64 ? 64
                                        : kAccCols <= 128 ? 128 : 256;
  static constexpr uint32_t kOffS = kOffP + (W16 ? kWStages : PW_PSTAGES) * PW_P_BYTES;  // group-scale ring
  static constexpr uint32_t kOffBar = kOffS + (W16 ? 0 : PW_PSTAGES * PW_S_BYTES);
  static constexpr uint32_t kSmem = kOffBar + 1024 + 1024;                   // barriers + alignment slack
  static_assert(kB % 1024 == 0, "token tiles keep 1 KiB alignment for the 128-byte swizzle");
  static_assert(kAStages >= 2 * PW_SUB, "the TMEM weight ring holds at least two code groups (one converting, one draining)");
  static_assert((uint32_t)PW_ROWS * TN * 4 <= kOffP, "split-K partial fits over the low-rank and token rings");
  static_assert(kSmem <= 227 * 1024, "shared memory per CTA");
};

struct PwBars {
  uint64_t full_p[PW_PSTAGES];   // code group and its scales landed (TMA bytes)
  uint64_t empty_p[PW_PSTAGES];  // code group read (one arrival per converter warp)
  uint64_t full_b[16];           // token tile (and, for a low-rank stage, its A) landed (TMA bytes)
  uint64_t empty_b[16];          // MMAs reading the token slot done (commit)
  uint64_t conv[12];             // TMEM weight stage written (one arrival per converter warp)
  uint64_t empty_a[12];          // MMAs reading the TMEM weight stage done (commit)
  uint64_t empty_l[PW_LSTAGES];  // MMAs reading the low-rank A slot done (commit)
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(PwBars) <= 1024, "barrier block");

struct PwArgs {
  const __half* scales16;  // fp16 group scales in tile order (svdq_prepare_packed)
  const __nv_bfloat16* bias;
  void* out;
  int64_t ldo;
  int M, N;
  int n_k, n_lr;   // residual and low-rank stages
  int spg;         // scales per row per code group: 256 / w_group
  int ks;          // CTAs per cluster along K
  int units_n;     // 128-row weight tiles
  int* err;
};

enum : int {
  kPwWaitPackedEmpty = 0x5101,
  kPwWaitTileEmpty = 0x5102,
  kPwWaitLowrankEmpty = 0x5103,
  kPwWaitConvPacked = 0x5201,
  kPwWaitConvEmpty = 0x5202,
  kPwWaitMmaTile = 0x5301,
  kPwWaitMmaConv = 0x5302,
  kPwWaitMmaDrain = 0x5303,
  kPwWaitEpilogue = 0x5401,
};

__device__ __forceinline__ uint32_t h2_sub(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t h2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint2 ld_shared_u2(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t ld_shared_u16(uint32_t addr) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}
// Contiguous global -> shared copy counted on an mbarrier (16-byte aligned, size a multiple of 16).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
__device__ __forceinline__ float ld_dsmem_f32(uint32_t cluster_addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(cluster_addr) : "memory");
  return v;
}
__device__ __forceinline__ void mbar_arrive_cta(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Eight codes of one native-order word -> four fp16x2 pairs (k0 k1, k2 k3, k4 k5, k6 k7), exact.
__device__ __forceinline__ void convert_word(uint32_t w, uint32_t s_lo, uint32_t s_hi, uint32_t* o) {
  constexpr uint32_t kExp = 0x64006400u;    // fp16x2 {1024, 1024}
  constexpr uint32_t kOffLo = 0x64086408u;  // {1032, 1032}: 1024 + the nibble offset 8
  constexpr uint32_t kOffHi = 0x64806480u;  // {1152, 1152}: 1024 + 16 * 8
  const uint32_t w8 = w >> 8;
  o[0] = h2_mul(h2_sub((w & 0x000F000Fu) | kExp, kOffLo), s_lo);
  o[1] = h2_mul(h2_sub((w & 0x00F000F0u) | kExp, kOffHi), s_hi);
  o[2] = h2_mul(h2_sub((w8 & 0x000F000Fu) | kExp, kOffLo), s_lo);
  o[3] = h2_mul(h2_sub((w8 & 0x00F000F0u) | kExp, kOffHi), s_hi);
}

template <int TN, bool OUT_F32, bool W16 = false>
__global__ void __launch_bounds__(PwLayout<TN, W16>::kThreads, PwLayout<TN, W16>::kTwoPerSm ? 2 : 1)
    packed_gemm_kernel(const __grid_constant__ CUtensorMap tm_a16, const __grid_constant__ CUtensorMap tm_codes,
                       const __grid_constant__ CUtensorMap tm_mid, const __grid_constant__ CUtensorMap tm_up,
                       const PwArgs args) {
  using L = PwLayout<TN, W16>;
  constexpr int AS = L::kAStages, BS = L::kBStages, WS = L::kWStages > 0 ? L::kWStages : 1;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  PwBars* bars = reinterpret_cast<PwBars*>(gbase + L::kOffBar);
  volatile int* abort_flag = &bars->abort_flag;
  const uint32_t l_ring = base + L::kOffL, b_ring = base + L::kOffB, p_ring = base + L::kOffP,
                 s_ring = base + L::kOffS;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ks = args.ks;
  const int crank = (int)(blockIdx.x % (unsigned)ks);
  const int unit = (int)(blockIdx.x / (unsigned)ks);
  const int nb = unit % args.units_n, mb = unit / args.units_n;
  const int n0 = nb * PW_ROWS, m0 = mb * TN;
  // K ranges are whole code groups (4 stages of 64 k); only the layer's last group may be short
  const int n_grp = (args.n_k + PW_SUB - 1) / PW_SUB;
  const int g0 = (int)((int64_t)crank * n_grp / ks), g1 = (int)((int64_t)(crank + 1) * n_grp / ks);
  const int kb0 = g0 * PW_SUB, kb1 = min(g1 * PW_SUB, args.n_k);
  const int n_res = kb1 - kb0;
  const int n_groups = g1 - g0;
  const int iters = n_res + (crank == ks - 1 ? args.n_lr : 0);

  auto bar = [&](const uint64_t& b) { return smem_u32(&b); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < PW_PSTAGES; ++s) {
      mbar_init(bar(bars->full_p[s]), 1);
      mbar_init(bar(bars->empty_p[s]), PW_CONV_WARPS);
    }
    for (int s = 0; s < BS; ++s) {
      mbar_init(bar(bars->full_b[s]), 1);
      mbar_init(bar(bars->empty_b[s]), 1);
    }
    for (int s = 0; s < AS; ++s) {
      mbar_init(bar(bars->conv[s]), W16 ? 1 : PW_CONV_WARPS);  // W16: the weight ring's TMA bytes
      mbar_init(bar(bars->empty_a[s]), 1);
    }
    for (int s = 0; s < PW_LSTAGES; ++s) mbar_init(bar(bars->empty_l[s]), 1);
    mbar_init(bar(bars->mma_done), 1);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tma_desc(&tm_a16);
    prefetch_tma_desc(&tm_codes);
    if (args.n_lr > 0) {
      prefetch_tma_desc(&tm_mid);
      prefetch_tma_desc(&tm_up);
    }
  }
  if (warp == 1) {
    tmem_alloc_1(smem_u32(&bars->tmem_base), L::kTmemCols);
    tmem_relinquish_1();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  pdl_wait();  // operands may come from the previous kernel on the stream
  pdl_trigger();

  if (warp == 0 && W16) {
    if (lane == 0) {
      // ------------------------------------------------ fp16 weight tiles: 128 rows x 64 k per stage
      // (tm_codes maps the fp16 weight here; conv / empty_a are the ring's full / empty barriers)
      uint32_t filled = 0, par = 0;
      bool ok = true;
      for (int it = 0; it < n_res && ok; ++it) {
        const int ws = it % WS;
        const uint32_t ph = (uint32_t)(it / WS) & 1u;
        if (!(ok = mbar_spin_wait(bar(bars->empty_a[ws]), ph ^ 1u, abort_flag, args.err, kPwWaitPackedEmpty))) break;
        mbar_arrive_expect_tx(bar(bars->conv[ws]), PW_P_BYTES);
        tma_load_2d(p_ring + (uint32_t)ws * PW_P_BYTES, &tm_codes, bar(bars->conv[ws]), (kb0 + it) * PW_KB, n0);
        filled |= 1u << ws;
        par = (par & ~(1u << ws)) | (ph << ws);
      }
      if (!ok)
        for (int ws = 0; ws < WS; ++ws)
          if (filled & (1u << ws)) mbar_wait_drain(bar(bars->conv[ws]), (par >> ws) & 1u, 100000000ull);
    }
  } else if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ packed codes: one 128-row x 256-k group per box
      uint32_t filled = 0, par = 0;
      bool ok = true;
      for (int it = 0; it < n_groups && ok; ++it) {
        const int s = it % PW_PSTAGES;
        const uint32_t ph = (uint32_t)(it / PW_PSTAGES) & 1u;
        if (!(ok = mbar_spin_wait(bar(bars->empty_p[s]), ph ^ 1u, abort_flag, args.err, kPwWaitPackedEmpty))) break;
        const uint32_t sbytes = (uint32_t)(PW_ROWS * args.spg * 2);
        mbar_arrive_expect_tx(bar(bars->full_p[s]), PW_P_BYTES + sbytes);
        tma_load_2d(p_ring + (uint32_t)s * PW_P_BYTES, &tm_codes, bar(bars->full_p[s]), (g0 + it) * (PW_SUB * PW_KB / 2),
                    n0);
        bulk_load(s_ring + (uint32_t)s * PW_S_BYTES,
                  args.scales16 + ((int64_t)nb * n_grp + g0 + it) * PW_ROWS * args.spg, sbytes, bar(bars->full_p[s]));
        filled |= 1u << s;
        par = (par & ~(1u << s)) | (ph << s);
      }
      if (!ok)
        for (int s = 0; s < PW_PSTAGES; ++s)
          if (filled & (1u << s)) mbar_wait_drain(bar(bars->full_p[s]), (par >> s) & 1u, 100000000ull);
    }
  } else if (warp == 2) {
    if (lane == 0) {
      // ------------------------------------------------ token tiles (+ low-rank A)
      uint32_t filled = 0, par = 0;
      bool ok = true;
      for (int it = 0; it < iters && ok; ++it) {
        const int s = it % BS;
        const uint32_t ph = (uint32_t)(it / BS) & 1u;
        if (!(ok = mbar_spin_wait(bar(bars->empty_b[s]), ph ^ 1u, abort_flag, args.err, kPwWaitTileEmpty))) break;
        const uint32_t fb = bar(bars->full_b[s]);
        const uint32_t bdst = b_ring + (uint32_t)s * L::kB;
        if (it < n_res) {
          mbar_arrive_expect_tx(fb, L::kB);
          tma_load_2d(bdst, &tm_a16, fb, (kb0 + it) * PW_KB, m0);
        } else {
          const int j = it - n_res, ls = j % PW_LSTAGES;
          const uint32_t lph = (uint32_t)(j / PW_LSTAGES) & 1u;
          if (!(ok = mbar_spin_wait(bar(bars->empty_l[ls]), lph ^ 1u, abort_flag, args.err, kPwWaitLowrankEmpty))) break;
          mbar_arrive_expect_tx(fb, L::kB + PW_A_BYTES);
          tma_load_2d(l_ring + (uint32_t)ls * PW_A_BYTES, &tm_up, fb, j * PW_KB, n0);
          tma_load_2d(bdst, &tm_mid, fb, j * PW_KB, m0);
        }
        filled |= 1u << s;
        par = (par & ~(1u << s)) | (ph << s);
      }
      if (!ok)
        for (int s = 0; s < BS; ++s)
          if (filled & (1u << s)) mbar_wait_drain(bar(bars->full_b[s]), (par >> s) & 1u, 100000000ull);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issue
      const uint32_t idesc_res = make_idesc(0u /*f16*/, 0u, PW_ROWS, TN);
      const uint32_t idesc_lr = make_idesc(kFmtBF16, kFmtBF16, PW_ROWS, TN);
      bool ok = true;
      for (int it = 0; it < iters && ok; ++it) {
        const int bs = it % BS;
        const uint32_t bph = (uint32_t)(it / BS) & 1u;
        if (!(ok = mbar_spin_wait(bar(bars->full_b[bs]), bph, abort_flag, args.err, kPwWaitMmaTile))) break;
        const uint64_t db = desc_k_sw128(b_ring + (uint32_t)bs * L::kB);
        if (W16 && it < n_res) {
          // fp16 weight stage from the shared-memory ring
          const int ws = it % WS;
          if (!(ok = mbar_spin_wait(bar(bars->conv[ws]), (uint32_t)(it / WS) & 1u, abort_flag, args.err,
                                    kPwWaitMmaConv)))
            break;
          tc_fence_after();
          const uint64_t da = desc_k_sw128(p_ring + (uint32_t)ws * PW_P_BYTES);
#pragma unroll
          for (int kk = 0; kk < PW_KB / 16; ++kk)
            umma_f16_1(tmem, da + (uint64_t)(kk * 2), db + (uint64_t)(kk * 2), idesc_res, (it > 0 || kk > 0) ? 1u : 0u);
          umma_commit_1(bar(bars->empty_a[ws]));
        } else if (it < n_res) {
          // a code group's stages are published together and released together, on the barriers
          // of the group's last TMEM slot (one wait and one commit per group, not per stage)
          const int as = it % AS;
          const int gi = it / PW_SUB;
          const int gslot = (gi * PW_SUB + PW_SUB - 1) % AS;
          if (it % PW_SUB == 0) {
            if (!(ok = mbar_spin_wait(bar(bars->conv[gslot]), (uint32_t)(gi / (AS / PW_SUB)) & 1u, abort_flag,
                                      args.err, kPwWaitMmaConv)))
              break;
            tc_fence_after();
          }
          const uint32_t ta = tmem + L::kAccCols + (uint32_t)as * PW_STAGE_COLS;
#pragma unroll
          for (int kk = 0; kk < PW_KB / 16; ++kk)
            umma_f16_1_tmem_a(tmem, ta + (uint32_t)(kk * 8), db + (uint64_t)(kk * 2), idesc_res,
                              (it > 0 || kk > 0) ? 1u : 0u);
          if (it % PW_SUB == PW_SUB - 1 || it == n_res - 1) umma_commit_1(bar(bars->empty_a[gslot]));
        } else {
          const int ls = (it - n_res) % PW_LSTAGES;
          tc_fence_after();
          const uint64_t da = desc_k_sw128(l_ring + (uint32_t)ls * PW_A_BYTES);
#pragma unroll
          for (int kk = 0; kk < PW_KB / 16; ++kk)
            umma_f16_1(tmem, da + (uint64_t)(kk * 2), db + (uint64_t)(kk * 2), idesc_lr, (it > 0 || kk > 0) ? 1u : 0u);
          umma_commit_1(bar(bars->empty_l[ls]));
        }
        umma_commit_1(bar(bars->empty_b[bs]));
      }
      // the epilogue reads the accumulator after every issued MMA has completed; this thread also
      // waits for that, so no MMA is in flight when the CTA frees TMEM or exits
      umma_commit_1(bar(bars->mma_done));
      if (!mbar_wait_drain(bar(bars->mma_done), 0, 1000000000ull)) {
        *abort_flag = 1;
        atomicCAS(args.err, 0, kPwWaitMmaDrain);
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp >= 4) {
    // ------------------------------------------------ conversion: codes -> fp16 weights in TMEM
    // Four warps per TMEM lane quarter, each owning 16 of a stage's 64 k for its 32 rows.  Per code
    // group (up to 4 stages) a thread loads its four 8-byte pieces, converts them together and
    // stores them to the four TMEM stages.
    const int q = warp & 3;            // TMEM lane quarter this warp may access
    const int part = (warp - 4) >> 2;  // which 16 of a stage's 64 k
    const int row = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const uint32_t code_row = (uint32_t)row * 128u;
    const uint32_t r7 = (uint32_t)(row & 7);
    const int spg = args.spg, gshift = spg == 8 ? 5 : spg == 4 ? 6 : spg == 2 ? 7 : 8;  // log2(G)
    bool ok = true;
    for (int gi = 0; gi < (W16 ? 0 : n_groups) && ok; ++gi) {  // W16: nothing to convert
      const int ps = gi % PW_PSTAGES;
      const int it0 = gi * PW_SUB;                 // first stage of the group (CTA-relative)
      const int nsub = min(PW_SUB, n_res - it0);
      ok = wait_spin(bar(bars->full_p[ps]), (uint32_t)(gi / PW_PSTAGES) & 1u, abort_flag, args.err,
                     kPwWaitConvPacked);
      if (!(ok = __all_sync(0xffffffffu, ok))) break;  // the lanes of a warp leave together
      const uint32_t srow = s_ring + (uint32_t)ps * PW_S_BYTES + (uint32_t)(row * spg) * 2u;
      const uint32_t prow = p_ring + (uint32_t)ps * PW_P_BYTES + code_row + 8u * (uint32_t)(part & 1);
      uint2 pk[PW_SUB];
      uint32_t sb[PW_SUB];
#pragma unroll
      for (int j = 0; j < PW_SUB; ++j) {
        // 128-byte swizzle: 16-byte chunk c of row r sits at c ^ (r % 8); this piece is half of chunk 2j + part/2
        pk[j] = ld_shared_u2(prow + ((((uint32_t)(2 * j + (part >> 1))) ^ r7) << 4));
        sb[j] = ld_shared_u16(srow + (uint32_t)(((j * PW_KB + 16 * part) >> gshift) * 2));
      }
      uint32_t v[PW_SUB][8];
#pragma unroll
      for (int j = 0; j < PW_SUB; ++j) {
        const uint32_t s_lo = sb[j] | (sb[j] << 16);
        const uint32_t s16 = (uint32_t)__half_as_ushort(__hmul(__ushort_as_half((unsigned short)sb[j]),
                                                               __float2half_rn(0.0625f)));
        const uint32_t s_hi = s16 | (s16 << 16);
        convert_word(pk[j].x, s_lo, s_hi, v[j]);
        convert_word(pk[j].y, s_lo, s_hi, v[j] + 4);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive_cta(bar(bars->empty_p[ps]));  // every lane has consumed its codes
      // this group's TMEM slots are free once the MMAs of the group that used them last are done
      ok = wait_spin(bar(bars->empty_a[(it0 + PW_SUB - 1) % AS]), ((uint32_t)(gi / (AS / PW_SUB)) & 1u) ^ 1u,
                     abort_flag, args.err, kPwWaitConvEmpty);
      if (!(ok = __all_sync(0xffffffffu, ok))) break;
      tc_fence_after();
#pragma unroll
      for (int j = 0; j < PW_SUB; ++j)
        if (j < nsub)
          tmem_st8(tmem + lane_off + L::kAccCols + (uint32_t)((it0 + j) % AS) * PW_STAGE_COLS + 8u * (uint32_t)part,
                   v[j]);
      // publish the group at once (one arrival per warp on the barrier of its last TMEM slot): the
      // MMAs wait for nothing but the stores, whose drain is short next to converting a group
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cta(bar(bars->conv[(it0 + PW_SUB - 1) % AS]));
    }
    if (warp < 8) {
      // ---------------------------------------------- epilogue: TMEM -> registers -> out or partial
      const int erow = q * 32 + lane;
      const int n = n0 + erow;
      const uint32_t taddr = tmem + lane_off;
      const bool done = wait_spin(bar(bars->mma_done), 0, abort_flag, args.err, kPwWaitEpilogue) && !*abort_flag;
      if (__all_sync(0xffffffffu, done)) {
        tc_fence_after();
        float bias_v = 0.f;
        if (ks == 1 && args.bias && n < args.N) bias_v = __bfloat162float(args.bias[n]);
        float* part = reinterpret_cast<float*>(gbase);  // [TN][128] over the low-rank/token rings (all MMAs are done)
#pragma unroll 1
        for (int c0 = 0; c0 < TN; c0 += 16) {
          uint32_t v[16];
          tmem_ld16(taddr + (uint32_t)c0, v);
          tmem_ld_wait_regs16(v);
          if (ks > 1) {
#pragma unroll
            for (int e = 0; e < 16; ++e) part[(c0 + e) * PW_ROWS + erow] = __uint_as_float(v[e]);
          } else if (n < args.N) {
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const int m = m0 + c0 + e;
              if (m < args.M) {
                const float y = __uint_as_float(v[e]) + bias_v;
                if constexpr (OUT_F32) static_cast<float*>(args.out)[(int64_t)m * args.ldo + n] = y;
                else static_cast<__nv_bfloat16*>(args.out)[(int64_t)m * args.ldo + n] = __float2bfloat16_rn(y);
              }
            }
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
    const int rows = PW_ROWS / ks;
    const uint32_t part_local = base;
    for (int o = threadIdx.x; o < rows * TN; o += L::kThreads) {
      const int rl = o % rows, col = o / rows;
      const int row = crank * rows + rl;
      const int n = n0 + row, m = m0 + col;
      const uint32_t off = (uint32_t)(col * PW_ROWS + row) * 4u;
      float pv[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) pv[c] = c < ks ? ld_dsmem_f32(mapa_shared(part_local + off, (uint32_t)c)) : 0.f;
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
    tmem_dealloc_1(tmem, L::kTmemCols);
  }
}

// Native nibble order: natural word [k0 k1 k2 k3 k4 k5 k6 k7] (nibble i at bits 4i) ->
// [k0 k2 k4 k6 | k1 k3 k5 k7].
__global__ void prepare_codes_kernel(const uint32_t* __restrict__ in, uint32_t* __restrict__ out, int64_t words) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < words; i += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t w = in[i];
    uint32_t o = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) o |= ((w >> (4 * j)) & 0xFu) << ((j & 1) ? 16 + 4 * (j >> 1) : 4 * (j >> 1));
    out[i] = o;
  }
}

template <typename T>
__device__ __forceinline__ float scale_f32(T v);
template <>
__device__ __forceinline__ float scale_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float scale_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float scale_f32<float>(float v) { return v; }

// Group scales -> fp16 in the kernel's tile order: for each 128-row tile and each 256-k code group,
// [128 rows][256 / G scales] contiguous (rows past N and groups past K_pad are zero), so one bulk
// copy brings a code group's scales with its codes.  *inexact (when given) is set when a scale is
// not an fp16 value or its sixteenth is not: the kernel's weights then round the scale once more
// than fp16(q * s) does (relative error at most 2^-11 on the weights of such groups).
template <typename T>
__global__ void prepare_scales_kernel(const T* __restrict__ in, __half* __restrict__ out, int N, int nG, int n_grp,
                                      int spg, int* __restrict__ inexact) {
  const int64_t count = (int64_t)((N + PW_ROWS - 1) / PW_ROWS) * n_grp * PW_ROWS * spg;
  int bad = 0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
    const int j = (int)(i % spg);
    const int r = (int)((i / spg) % PW_ROWS);
    const int64_t tg = i / ((int64_t)spg * PW_ROWS);
    const int grp = (int)(tg % n_grp);
    const int n = (int)(tg / n_grp) * PW_ROWS + r;
    const int g = grp * spg + j;  // weight group along K
    __half h = __float2half_rn(0.f);
    if (n < N && g < nG) {
      const float s = scale_f32<T>(in[(int64_t)n * nG + g]);
      h = __float2half_rn(s);
      const __half h16 = __hmul(h, __float2half_rn(0.0625f));
      bad |= (__half2float(h) != s) || (__half2float(h16) * 16.0f != __half2float(h));
    }
    out[i] = h;
  }
  if (__syncthreads_or(bad) && threadIdx.x == 0 && inexact) atomicExch(inexact, 1);
}

// CTAs of one launch resident per SM: two for the fp16-weight mode with up to 64 tokens per tile.
int pw_ctas_per_sm(int tn, bool w16) { return w16 && tn <= 64 ? 2 : 1; }

struct PwPlan {
  int tn, ks, units_n, units_m;
};

// 256-token tiles put a 256-token batch into one wave of CTAs that each convert their weight
// tile once (128-token tiles: two waves, each converting every weight tile again).
int pick_tn(int M) { return M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256; }

// Split factor: among KS in {1, 2, 4, 8} (at least two code groups per CTA), the fewest waves of
// CTAs, then the fullest last wave; ties go to the smaller KS.  Each CTA has a fixed cost (set-up,
// pipeline fill, epilogue, cluster reduction), so an extra wave costs more than idle SMs.
PwPlan plan_packed(int M, int N, int K_pad, bool w16 = false) {
  PwPlan p;
  p.tn = pick_tn(M);
  p.units_n = (N + PW_ROWS - 1) / PW_ROWS;
  p.units_m = (M + p.tn - 1) / p.tn;
  const int n_k = K_pad / PW_KB;
  const long long units = (long long)p.units_n * p.units_m;
  const long long slots = (long long)num_sms() * pw_ctas_per_sm(p.tn, w16);
  p.ks = 1;
  double best = -1.0;
  long long best_waves = 1ll << 40;
  const int n_grp = (n_k + PW_SUB - 1) / PW_SUB;
  for (int ks = 1; ks <= 8 && (ks == 1 || n_grp / ks >= 2); ks *= 2) {
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

template <int TN, bool OUT_F32, bool W16 = false>
int launch_pw(const CUtensorMap& ta, const CUtensorMap& tc, const CUtensorMap& tmid, const CUtensorMap& tup,
              const PwArgs& a, int grid, cudaStream_t stream) {
  auto kern = packed_gemm_kernel<TN, OUT_F32, W16>;
  constexpr uint32_t smem = PwLayout<TN, W16>::kSmem;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return check_cuda(e, "svdq_packed_gemm: shared memory attribute");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(PwLayout<TN, W16>::kThreads, 1, 1);
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
  e = cudaLaunchKernelEx(&cfg, kern, ta, tc, tmid, tup, a);
  if (e != cudaSuccess) return check_cuda(e, "svdq_packed_gemm launch");
  return check_launch("svdq_packed_gemm launch");
}

template <bool OUT_F32, bool W16 = false>
int launch_pw_tn(int tn, const CUtensorMap& ta, const CUtensorMap& tc, const CUtensorMap& tmid, const CUtensorMap& tup,
                 const PwArgs& a, int grid, cudaStream_t stream) {
  switch (tn) {
    case 16: return launch_pw<16, OUT_F32, W16>(ta, tc, tmid, tup, a, grid, stream);
    case 32: return launch_pw<32, OUT_F32, W16>(ta, tc, tmid, tup, a, grid, stream);
    case 64: return launch_pw<64, OUT_F32, W16>(ta, tc, tmid, tup, a, grid, stream);
    case 128: return launch_pw<128, OUT_F32, W16>(ta, tc, tmid, tup, a, grid, stream);
    default: return launch_pw<256, OUT_F32, W16>(ta, tc, tmid, tup, a, grid, stream);
  }
}

}  // namespace

// The small-batch kernel (packed_small.cu): batches of up to kSmallBatchMax tokens.
constexpr int kSmallBatchMax = 64;
int packed_small_gemm(const void* act, bool i8, const float* ascales_t, int64_t lda_s, int a_group, const void* codes,
                      const void* scales16, int w_group, const void* mid_hl, const void* up_hl, int R2,
                      const void* bias, void* out, int out_dtype, int64_t ldo, int M, int N, int K_pad,
                      cudaStream_t stream);
int packed_small_plan(int M, int N, int K_pad, int* out4);

}  // namespace svdq

extern "C" int svdq_prepare_packed(const void* qweight, const void* scales, int scale_dtype, int N, int K_pad,
                                   int w_group, void* out_codes, void* out_scales16, int* inexact,
                                   cudaStream_t stream) {
  using namespace svdq;
  SVDQ_REQUIRE(qweight && scales && out_codes && out_scales16, "svdq_prepare_packed: null pointer");
  SVDQ_REQUIRE(N > 0 && K_pad > 0 && K_pad % 64 == 0, "svdq_prepare_packed: K_pad must be a positive multiple of 64");
  SVDQ_REQUIRE((w_group == 32 || w_group == 64 || w_group == 128 || w_group == 256) && K_pad % w_group == 0,
               "svdq_prepare_packed: w_group must be 32, 64, 128 or 256 and divide K_pad");
  SVDQ_REQUIRE((reinterpret_cast<uintptr_t>(qweight) & 3u) == 0 && (reinterpret_cast<uintptr_t>(out_codes) & 15u) == 0,
               "svdq_prepare_packed: qweight must be 4-byte and out_codes 16-byte aligned");
  const int64_t words = (int64_t)N * K_pad / 8;
  const int threads = 256;
  const unsigned blocks = (unsigned)std::min<int64_t>((words + threads - 1) / threads, (int64_t)num_sms() * 32);
  prepare_codes_kernel<<<blocks, threads, 0, stream>>>(static_cast<const uint32_t*>(qweight),
                                                       static_cast<uint32_t*>(out_codes), words);
  int st = check_launch("svdq_prepare_packed: codes");
  if (st) return st;
  const int nG = K_pad / w_group, n_grp = (K_pad + PW_GROUP_K - 1) / PW_GROUP_K, spg = PW_GROUP_K / w_group;
  const int64_t count = (int64_t)((N + PW_ROWS - 1) / PW_ROWS) * n_grp * PW_ROWS * spg;
  const unsigned sblocks = (unsigned)std::min<int64_t>((count + threads - 1) / threads, (int64_t)num_sms() * 8);
  __half* o = static_cast<__half*>(out_scales16);
  switch (scale_dtype) {
    case SVDQ_BF16:
      prepare_scales_kernel<<<sblocks, threads, 0, stream>>>(static_cast<const __nv_bfloat16*>(scales), o, N, nG, n_grp,
                                                             spg, inexact);
      break;
    case SVDQ_FP16:
      prepare_scales_kernel<<<sblocks, threads, 0, stream>>>(static_cast<const __half*>(scales), o, N, nG, n_grp, spg,
                                                             inexact);
      break;
    case SVDQ_FP32:
      prepare_scales_kernel<<<sblocks, threads, 0, stream>>>(static_cast<const float*>(scales), o, N, nG, n_grp, spg,
                                                             inexact);
      break;
    default:
      return set_error(SVDQ_ERR_INVALID_ARGUMENT, "svdq_prepare_packed: scale_dtype must be bf16, fp16 or fp32");
  }
  return check_launch("svdq_prepare_packed: scales");
}

extern "C" int svdq_packed_gemm_plan(int M, int N, int K_pad, int* out4) {
  using namespace svdq;
  SVDQ_REQUIRE(out4, "svdq_packed_gemm_plan: out4 is NULL");
  SVDQ_REQUIRE(M > 0 && N > 0 && K_pad > 0 && K_pad % 64 == 0, "svdq_packed_gemm_plan: bad M/N/K_pad");
  if (M <= kSmallBatchMax) return packed_small_plan(M, N, K_pad, out4);
  const PwPlan p = plan_packed(M, N, K_pad);
  out4[0] = p.tn;
  out4[1] = p.ks;
  out4[2] = p.units_n * p.units_m * p.ks;
  out4[3] = pw_ctas_per_sm(p.tn, false);
  return SVDQ_OK;
}

extern "C" int svdq_packed_gemm(const void* a16, const void* codes, const void* scales16, int w_group,
                                const void* mid_hl, const void* up_hl, int R2, const void* bias, void* out,
                                int out_dtype, int64_t ldo, int M, int N, int K_pad, cudaStream_t stream) {
  using namespace svdq;
  SVDQ_REQUIRE(a16 && codes && scales16 && out, "svdq_packed_gemm: null operand pointer");
  SVDQ_REQUIRE(M >= 0 && N > 0 && K_pad > 0 && K_pad % 64 == 0, "svdq_packed_gemm: bad M/N/K_pad");
  SVDQ_REQUIRE((w_group == 32 || w_group == 64 || w_group == 128 || w_group == 256) && K_pad % w_group == 0,
               "svdq_packed_gemm: w_group must be 32, 64, 128 or 256 and divide K_pad");
  SVDQ_REQUIRE((reinterpret_cast<uintptr_t>(scales16) & 15u) == 0, "svdq_packed_gemm: scales16 must be 16-byte aligned");
  SVDQ_REQUIRE(N % 8 == 0 && ldo >= N && ldo % 8 == 0, "svdq_packed_gemm: N and ldo must be multiples of 8, ldo >= N");
  SVDQ_REQUIRE(R2 >= 0 && R2 % 64 == 0, "svdq_packed_gemm: R2 must be a multiple of 64");
  SVDQ_REQUIRE(R2 == 0 || (mid_hl && up_hl), "svdq_packed_gemm: mid_hl/up_hl are NULL");
  SVDQ_REQUIRE(out_dtype == SVDQ_BF16 || out_dtype == SVDQ_FP32, "svdq_packed_gemm: out_dtype must be bf16 or fp32");
  SVDQ_REQUIRE(!bias || (reinterpret_cast<uintptr_t>(bias) & 1u) == 0, "svdq_packed_gemm: bias must be 2-byte aligned");
  if (M == 0) return SVDQ_OK;
  if (M <= kSmallBatchMax) {
    SVDQ_REQUIRE((reinterpret_cast<uintptr_t>(a16) & 15u) == 0 && (reinterpret_cast<uintptr_t>(codes) & 15u) == 0,
                 "svdq_packed_gemm: a16 and codes must be 16-byte aligned");
    return packed_small_gemm(a16, false, nullptr, 0, 0, codes, scales16, w_group, mid_hl, up_hl, R2, bias, out,
                             out_dtype, ldo, M, N, K_pad, stream);
  }
  int* err = device_error_word();
  if (!err) return set_error(SVDQ_ERR_CUDA, "svdq_packed_gemm: device error word unavailable");
  const PwPlan p = plan_packed(M, N, K_pad);
  CUtensorMap ta, tc, tmid, tup;
  int st;
  if ((st = make_tma_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a16, K_pad, M, (uint64_t)K_pad * 2, PW_KB, p.tn,
                        CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if ((st = make_tma_2d(&tc, CU_TENSOR_MAP_DATA_TYPE_UINT8, codes, K_pad / 2, N, (uint64_t)K_pad / 2,
                        PW_SUB * PW_KB / 2, PW_ROWS, CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if (R2 > 0) {
    if ((st = make_tma_2d(&tmid, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, mid_hl, R2, M, (uint64_t)R2 * 2, PW_KB, p.tn,
                          CU_TENSOR_MAP_SWIZZLE_128B)))
      return st;
    if ((st = make_tma_2d(&tup, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, up_hl, R2, N, (uint64_t)R2 * 2, PW_KB, PW_ROWS,
                          CU_TENSOR_MAP_SWIZZLE_128B)))
      return st;
  } else {
    tmid = ta;
    tup = ta;
  }
  PwArgs a;
  a.scales16 = static_cast<const __half*>(scales16);
  a.bias = static_cast<const __nv_bfloat16*>(bias);
  a.out = out;
  a.ldo = ldo;
  a.M = M;
  a.N = N;
  a.n_k = K_pad / PW_KB;
  a.n_lr = R2 / PW_KB;
  a.spg = PW_GROUP_K / w_group;
  a.ks = p.ks;
  a.units_n = p.units_n;
  a.err = err;
  const int grid = p.units_n * p.units_m * p.ks;
  return out_dtype == SVDQ_FP32 ? launch_pw_tn<true>(p.tn, ta, tc, tmid, tup, a, grid, stream)
                                : launch_pw_tn<false>(p.tn, ta, tc, tmid, tup, a, grid, stream);
}

extern "C" int svdq_linear_gemm_small(const void* a16, const void* w16, const void* mid_hl, const void* up_hl, int R2,
                                      const void* bias, void* out, int out_dtype, int64_t ldo, int M, int N, int K_pad,
                                      cudaStream_t stream) {
  using namespace svdq;
  SVDQ_REQUIRE(a16 && w16 && out, "svdq_linear_gemm_small: null operand pointer");
  SVDQ_REQUIRE(M >= 0 && N > 0 && K_pad > 0 && K_pad % 64 == 0, "svdq_linear_gemm_small: bad M/N/K_pad");
  SVDQ_REQUIRE((reinterpret_cast<uintptr_t>(a16) & 15u) == 0 && (reinterpret_cast<uintptr_t>(w16) & 15u) == 0,
               "svdq_linear_gemm_small: a16 and w16 must be 16-byte aligned");
  SVDQ_REQUIRE(N % 8 == 0 && ldo >= N && ldo % 8 == 0, "svdq_linear_gemm_small: N and ldo must be multiples of 8, ldo >= N");
  SVDQ_REQUIRE(R2 >= 0 && R2 % 64 == 0, "svdq_linear_gemm_small: R2 must be a multiple of 64");
  SVDQ_REQUIRE(R2 == 0 || (mid_hl && up_hl), "svdq_linear_gemm_small: mid_hl/up_hl are NULL");
  SVDQ_REQUIRE(out_dtype == SVDQ_BF16 || out_dtype == SVDQ_FP32,
               "svdq_linear_gemm_small: out_dtype must be bf16 or fp32");
  SVDQ_REQUIRE(!bias || (reinterpret_cast<uintptr_t>(bias) & 1u) == 0, "svdq_linear_gemm_small: bias must be 2-byte aligned");
  if (M == 0) return SVDQ_OK;
  int* err = device_error_word();
  if (!err) return set_error(SVDQ_ERR_CUDA, "svdq_linear_gemm_small: device error word unavailable");
  const PwPlan p = plan_packed(M, N, K_pad, true);
  CUtensorMap ta, tw, tmid, tup;
  int st;
  if ((st = make_tma_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a16, K_pad, M, (uint64_t)K_pad * 2, PW_KB, p.tn,
                        CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if ((st = make_tma_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, w16, K_pad, N, (uint64_t)K_pad * 2, PW_KB, PW_ROWS,
                        CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if (R2 > 0) {
    if ((st = make_tma_2d(&tmid, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, mid_hl, R2, M, (uint64_t)R2 * 2, PW_KB, p.tn,
                          CU_TENSOR_MAP_SWIZZLE_128B)))
      return st;
    if ((st = make_tma_2d(&tup, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, up_hl, R2, N, (uint64_t)R2 * 2, PW_KB, PW_ROWS,
                          CU_TENSOR_MAP_SWIZZLE_128B)))
      return st;
  } else {
    tmid = ta;
    tup = ta;
  }
  PwArgs a;
  a.scales16 = nullptr;  // the fp16 weight already holds q * s
  a.bias = static_cast<const __nv_bfloat16*>(bias);
  a.out = out;
  a.ldo = ldo;
  a.M = M;
  a.N = N;
  a.n_k = K_pad / PW_KB;
  a.n_lr = R2 / PW_KB;
  a.spg = 1;
  a.ks = p.ks;
  a.units_n = p.units_n;
  a.err = err;
  const int grid = p.units_n * p.units_m * p.ks;
  return out_dtype == SVDQ_FP32 ? launch_pw_tn<true, true>(p.tn, ta, tw, tmid, tup, a, grid, stream)
                                : launch_pw_tn<false, true>(p.tn, ta, tw, tmid, tup, a, grid, stream);
}
