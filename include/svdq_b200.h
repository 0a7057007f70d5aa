/*
 * svdq_b200.h -- C ABI of the B200 (sm_100a) SVDQuant linear runtime.
 *
 * Plain pointers, sizes and a cudaStream_t; no framework types.  Every entry
 * point is asynchronous on the given stream unless stated otherwise and
 * returns an int status (SVDQ_OK on success).  Device pointers are borrowed
 * for the duration of the call only.  A failing call never falls back to
 * another implementation: it returns an error status, and svdq_last_error()
 * gives a one-line reason for the calling host thread.
 *
 * The linear forward is two launches:
 *   activation pass  svdq_act_quant (W4A4) or svdq_w4a16_prep (W4A16)
 *   GEMM             svdq_linear_gemm
 * on operands prepared once per layer by svdq_repack_weight and
 * svdq_build_up_hl.
 *
 * Data layouts (row-major unless stated; K_pad is the checkpoint's padded input
 * width, 2 * qweight.shape[1]):
 *   x            [M, K_in]        bf16, row stride ldx elements
 *   smooth       [K_in]           bf16
 *   l2           [rank, K_in]     bf16
 *   lora_down    [lora_rank, K_in] bf16 (all adapters stacked)
 *   lora_col_scale [lora_rank]    fp32 (adapter multiplier per stacked row)
 *   act packed   [M, K_pad/2]     u8, nibble = q + 8, even k in the low nibble
 *   act scales   [M, K_pad/a_group] bf16
 *   a16          [M, K_pad]       fp16 GEMM operand: q * scale (W4A4, exact) or
 *                                 x / smooth (W4A16)
 *   mid_hl       [M, R2]          bf16: [hi(r_tot) | lo(r_tot) | 0], r_tot = rank + lora_rank,
 *                                 hi = bf16(mid), lo = bf16(mid - hi), R2 = round_up(2 r_tot, 64)
 *   up_hl        [N, R2]          bf16: [up(r_tot) | up(r_tot) | 0], up = [l1 | lora_up]
 *   w16          [N, K_pad]       fp16 GEMM operand: q_w * weight scale
 *   out          [M, N]           bf16 or fp32, row stride ldo elements
 */
#ifndef SVDQ_B200_H
#define SVDQ_B200_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

enum svdq_status {
  SVDQ_OK = 0,
  SVDQ_ERR_INVALID_ARGUMENT = 1, /* shapes, strides, alignment, null pointers */
  SVDQ_ERR_UNSUPPORTED = 2,      /* valid request outside what the kernels implement */
  SVDQ_ERR_CUDA = 3,             /* a CUDA runtime / driver call failed */
  SVDQ_ERR_TIMEOUT = 4,          /* a bounded host-side wait ran out */
  SVDQ_ERR_DEVICE_WAIT = 5       /* a bounded in-kernel wait ran out (see svdq_device_error) */
};

enum svdq_dtype { SVDQ_BF16 = 0, SVDQ_FP16 = 1, SVDQ_FP32 = 2 };

/* Epilogue operations of svdq_linear_gemm_epi: y = the linear's output, z = the operand. */
enum svdq_epilogue {
  SVDQ_EPI_NONE = 0,
  SVDQ_EPI_ADD = 1,          /* z + y            residual add                        */
  SVDQ_EPI_SIGMOID_MUL = 2,  /* z * sigmoid(y)   output gated by this linear         */
  SVDQ_EPI_SILU_MUL = 3      /* silu(z) * y      gated MLP, z the gate linear's output */
};

/* One-line description of the last failure on this host thread. */
const char* svdq_last_error(void);
/* Library version string ("svdq_b200 <major>.<minor>"). */
const char* svdq_version(void);

/*
 * In-kernel bounded waits record the place they gave up in a device-side
 * word instead of hanging.  Reads (and optionally clears) that word on the
 * current device; synchronizes the device.  *code == 0 means no failure.
 * Codes: 0x101-0x303 GEMM waits (0x302: a split tile's owner waited for a
 * partial), 0x41xx activation-pass waits, 0x4200 an
 * activation group scale above 65504/7 (the fp16 GEMM operand a16 overflowed),
 * 0x7E01 the diagnostic wait below; the first failure since the last clear is kept.
 */
int svdq_device_error(int* code, int clear);

/*
 * Diagnostic for the bounded-wait machinery: one CTA waits on an mbarrier that
 * nothing completes, with an in-kernel limit of limit_us microseconds
 * (1 .. 5,000,000).  The wait gives up, records 0x7E01 in the device error
 * word and the kernel exits; the CUDA context stays usable.  Asynchronous on
 * `stream`; read the result with svdq_device_error.
 */
int svdq_selftest_bounded_wait(int limit_us, cudaStream_t stream);

/*
 * Diagnostic for the GEMM epilogue's activations: out[i] = bf16(sigmoid(in[i])) for
 * SVDQ_EPI_SIGMOID_MUL or bf16(silu(in[i])) for SVDQ_EPI_SILU_MUL, computed by the device code
 * svdq_linear_gemm_epi uses for bf16 output (fast instructions with an exact fallback near bf16
 * rounding midpoints).  in / out: n bf16 values.  Lets a test compare it with torch.sigmoid /
 * torch.nn.functional.silu over every bf16 input.
 */
int svdq_selftest_epilogue_act(int epilogue, const void* in, void* out, int n, cudaStream_t stream);

/*
 * Device workspace (bytes) the activation passes need for the low-rank
 * down-projection: the fp32 partial sums of the K slices, which a second
 * launch of the same call adds in slice order (deterministic) into mid_hl.
 * 256-byte aligned; needs no clearing (every slice writes all of its partials
 * before the second launch reads them).  One call at a time per workspace
 * (calls ordered on one stream are fine).  0 when rank + lora_rank == 0 or mid
 * is not requested.
 */
size_t svdq_act_quant_workspace_bytes(int M, int K_pad, int rank, int lora_rank);

/*
 * Activation pass of the W4A4 linear.  Replaces, on the device, the reference's
 *   x_hat = x / smooth                                  (src/krea2_svdquant/quant/svd.py:122)
 *   quantize_symmetric_int4(x_hat, a_group) + pack_int4 (src/krea2_svdquant/quant/pack.py:6-56)
 *   F.linear(x_hat, l2)                                 (svd.py:159, low-rank down)
 *   F.linear(x, lora_down) * multiplier                 (src/krea2_svdquant/runtime/linear.py:38-45)
 * in one pass over x.  Codes, packing and scales are bit-exact with the
 * reference for every finite input: x / smooth and x_hat / scale follow IEEE
 * division (a fast correctly rounded quotient where it is proven equal, IEEE
 * division for tiny x, huge quotients and non-normal smoothing factors).
 * a16 = q * scale is exact while every group scale lies in
 * [2^-17, 65504/7] (group max |x_hat| up to ~65000); larger scales overflow
 * fp16 and are reported through svdq_device_error (code 0x4200).  Optional
 * outputs may be NULL: out_packed / out_scales (the
 * reference-format codes), out_a16 (the GEMM operand), out_mid_hl (needs
 * rank + lora_rank > 0 and a workspace of svdq_act_quant_workspace_bytes(),
 * zero-filled before its first use as described there).
 * out_packed and out_scales are written together (both NULL or both set).
 *   a_group in {64, 128}; K_in <= K_pad; K_pad % 64 == 0; K_pad % a_group == 0;
 *   K_in % 8 == 0; rank % 8 == 0, lora_rank % 8 == 0, rank + lora_rank <= 256;
 *   ldx % 8 == 0; all pointers 16-byte aligned.
 */
int svdq_act_quant(const void* x, int64_t ldx, const void* smooth,
                   const void* l2, int rank,
                   const void* lora_down, const float* lora_col_scale, int lora_rank,
                   int M, int K_in, int K_pad, int a_group,
                   void* out_packed, void* out_scales, void* out_a16,
                   void* out_mid_hl, int R2,
                   void* workspace, size_t workspace_bytes, cudaStream_t stream);

/*
 * svdq_act_quant for the int8-code GEMM (svdq_w4a4_gemm): the same quantization (codes and scales
 * bit-exact with quantize_symmetric_int4, src/krea2_svdquant/quant/pack.py:6-23), written as
 *   out_codes8    [M, K_pad] int8: q in [-8, 7] (the unpacked form of pack_int4's codes);
 *   out_ascales_t [K_pad / a_group, lda_s] fp32: the bf16 group scales, group-major (row g holds
 *                 the scales of group g for tokens 0..M-1; tokens M..round_up(M, 64)-1 below
 *                 lda_s are written as zero), lda_s >= M;
 * plus out_mid_hl as svdq_act_quant writes it (same workspace rules).  No a16 is written.
 *   out_codes8 and out_ascales_t 16-byte aligned; other requirements as svdq_act_quant.
 */
int svdq_act_quant_i8(const void* x, int64_t ldx, const void* smooth,
                      const void* l2, int rank,
                      const void* lora_down, const float* lora_col_scale, int lora_rank,
                      int M, int K_in, int K_pad, int a_group,
                      void* out_codes8, float* out_ascales_t, int64_t lda_s,
                      void* out_mid_hl, int R2,
                      void* workspace, size_t workspace_bytes, cudaStream_t stream);

/*
 * svdq_act_quant without a workspace argument: allocates nothing.  No
 * counterpart in the reference (its activation quantization runs in torch /
 * Triton and allocates through the framework).  For callers that cannot
 * allocate device memory at the call site (an FFI host whose device memory is
 * owned by another framework; a serving loop that forbids allocation after
 * warm-up).  The K-slice scratch is a file-scope device array of
 * svdq_act_quant_noalloc_scratch_bytes() (8 MiB) per device; a call needing
 * more (svdq_act_quant_workspace_bytes() > 8 MiB) returns
 * SVDQ_ERR_UNSUPPORTED.  The scratch needs no clearing (the workspace contract
 * above), and each call leaves its partial sums in it.  The scratch address is looked up with
 * cudaGetSymbolAddress on the first call in each CUDA context (the device's
 * primary context or another context the host made current), whatever that
 * call's arguments: if that first call would fall inside a stream capture,
 * make one call of any shape before capturing.  All calls on a device share
 * the scratch: calls that overlap in time race and must be serialized by the
 * caller.  Arguments and results otherwise as
 * svdq_act_quant.
 */
size_t svdq_act_quant_noalloc_scratch_bytes(void);
int svdq_act_quant_noalloc(const void* x, int64_t ldx, const void* smooth,
                           const void* l2, int rank,
                           const void* lora_down, const float* lora_col_scale, int lora_rank,
                           int M, int K_in, int K_pad, int a_group,
                           void* out_packed, void* out_scales, void* out_a16,
                           void* out_mid_hl, int R2, cudaStream_t stream);

/*
 * Activation pass of the W4A16 linear: a16 = fp16(fp32(x) / fp32(smooth)) and
 * the low-rank/LoRA down-projection.  Replaces x / smooth and F.linear(x_hat, l2)
 * of the reference's float run (svd.py:122, 159) and the smoothing done by
 * kernels/triton/generic_int4.py:169-191.  l2_f16 is l2 [rank, K_in] in fp16
 * (converted once at load; the product x_hat @ l2^T runs on fp16 MMAs).
 * Same constraints as svdq_act_quant.
 */
int svdq_w4a16_prep(const void* x, int64_t ldx, const void* smooth,
                    const void* l2_f16, int rank,
                    const void* lora_down, const float* lora_col_scale, int lora_rank,
                    int M, int K_in, int K_pad,
                    void* out_a16, void* out_mid_hl, int R2,
                    void* workspace, size_t workspace_bytes, cudaStream_t stream);

/*
 * Load-time weight preparation: packed INT4 qweight [N, K_pad/2] + group scales
 * [N, K_pad/w_group] (bf16, fp16 or fp32 as the checkpoint stores them) ->
 * w16 [N, K_pad] fp16 = q * scale (exact for bf16 scales).  Replaces the
 * per-call unpack + dequantize of the reference (src/krea2_svdquant/quant/svd.py:128-135,
 * quant/pack.py:26-70); reads the layout load_svdquant_transformer reads
 * (src/krea2_svdquant/runtime/load.py:104-124).
 */
int svdq_repack_weight(const void* qweight, const void* scales, int scale_dtype,
                       int N, int K_pad, int w_group, void* out_w16, cudaStream_t stream);

/*
 * Build up_hl [N, R2] = [up | up | 0] from up = [l1 | lora_up] (bf16 inputs).
 * l1 [N, rank], lora_up [N, lora_rank] (may be NULL when lora_rank == 0).
 * The low-rank up-projection operand of svd.py:159 and linear.py:45.
 */
int svdq_build_up_hl(const void* l1, int rank, const void* lora_up, int lora_rank,
                     int N, void* out_up_hl, int R2, cudaStream_t stream);

/*
 * SVDQuant linear GEMM with the fused low-rank/LoRA up-projection and bias:
 *   out[m, n] = sum_k a16[m,k] w16[n,k] + sum_j mid_hl[m,j] up_hl[n,j] + bias[n]
 * tcgen05 MMAs on CTA pairs, fp32 accumulation in TMEM, bias and output cast
 * in the epilogue.  Replaces F.linear(x_hat, w_res) + F.linear(mid, l1) + bias
 * of src/krea2_svdquant/quant/svd.py:158-162 (W4A4 form: README.md:64; the
 * slot of kernels/gluon/blackwell_fused_svdquant.py:29-38 and of the Triton
 * kernels in kernels/triton/generic_int4.py:19-133).
 *   K_pad % 64 == 0, N % 8 == 0, ldo % 8 == 0, R2 % 64 == 0 (R2 may be 0),
 *   out_dtype in {SVDQ_BF16, SVDQ_FP32}; bias may be NULL (16-byte aligned).
 */
int svdq_linear_gemm(const void* a16, const void* w16,
                     const void* mid_hl, const void* up_hl, int R2,
                     const void* bias,
                     void* out, int out_dtype, int64_t ldo,
                     int M, int N, int K_pad,
                     cudaStream_t stream);

/*
 * svdq_linear_gemm for small batches, swap-AB: the weight rows are the tcgen05 MMA's M (128 per
 * CTA) and the tokens its N (16 to 256 per tile), so a 16-token batch runs 128x16 MMAs instead
 * of 256x256 tiles that are mostly padding, and the layer is bound by the bytes of w16 rather
 * than by MMAs.  Same computation, operands and output as svdq_linear_gemm; the fp32 summation
 * order differs (split K over clusters of 2-8 CTAs when the tiles would leave SMs idle, summed in
 * a fixed order, so results are deterministic).  The slot of the reference's small-batch Triton
 * path (kernels/triton/generic_int4.py:19-133).
 *   a16 and w16 16-byte aligned; K_pad % 64 == 0, N % 8 == 0, ldo % 8 == 0, R2 % 64 == 0;
 *   out_dtype in {SVDQ_BF16, SVDQ_FP32}; bias may be NULL.  Any M; meant for M <= 256.
 */
int svdq_linear_gemm_small(const void* a16, const void* w16,
                           const void* mid_hl, const void* up_hl, int R2,
                           const void* bias,
                           void* out, int out_dtype, int64_t ldo,
                           int M, int N, int K_pad,
                           cudaStream_t stream);

/*
 * Bytes of the split-tail workspace of svdq_linear_gemm_ws on the current
 * device (sync words plus one fp32 256x128 partial tile per CTA of a full grid).
 */
size_t svdq_linear_gemm_workspace_bytes(void);

/*
 * svdq_linear_gemm with a workspace.  When the output tiles leave a last wave
 * that would keep most CTA pairs idle, that wave's K iterations are split into
 * equal ranges over all pairs; the pair holding the start of a tile adds the
 * other ranges' fp32 partials in K order, so results are deterministic (for a
 * given shape and device) but differ from svdq_linear_gemm in fp32 summation
 * order.  Same computation and arguments as svdq_linear_gemm otherwise.
 *   workspace: 256-byte aligned, at least svdq_linear_gemm_workspace_bytes(),
 *   ZERO-FILLED before its first use; each launch leaves it ready for the next.
 *   One launch at a time per workspace (launches ordered on one stream are
 *   fine).  workspace == NULL gives svdq_linear_gemm.
 */
int svdq_linear_gemm_ws(const void* a16, const void* w16,
                        const void* mid_hl, const void* up_hl, int R2,
                        const void* bias,
                        void* out, int out_dtype, int64_t ldo,
                        int M, int N, int K_pad,
                        void* workspace, size_t workspace_bytes,
                        cudaStream_t stream);

/*
 * svdq_linear_gemm_ws whose epilogue also applies one elementwise operation
 * with an operand z [M, N] (out_dtype, row stride ld_aux): z + y, z * sigmoid(y)
 * or silu(z) * y, y being the linear's output (enum svdq_epilogue).  With bf16
 * output, y and the activation are rounded to bf16 before the combining
 * operation, so the result equals the unfused sequence of bf16 tensor ops
 * (linear, then sigmoid / silu, then the product or sum).  Replaces the glue
 * that follows the linears of a transformer block (the gate products and the
 * residual adds around runtime/linear.py:148-161's forward), saving one
 * round trip of y through HBM per operation.
 *   aux: 16-byte aligned, ld_aux >= N, ld_aux % 8 == 0; it may be out itself
 *   (with ld_aux == ldo): every element is read before the same thread writes
 *   it.  SVDQ_EPI_NONE ignores aux.  Other arguments as svdq_linear_gemm_ws.
 */
int svdq_linear_gemm_epi(const void* a16, const void* w16,
                         const void* mid_hl, const void* up_hl, int R2,
                         const void* bias,
                         int epilogue, const void* aux, int64_t ld_aux,
                         void* out, int out_dtype, int64_t ldo,
                         int M, int N, int K_pad,
                         void* workspace, size_t workspace_bytes,
                         cudaStream_t stream);

/*
 * One GEMM of a grouped launch (svdq_linear_gemm_group): the operands and output of one
 * svdq_linear_gemm_epi call, with the dimensions the group shares taken out.
 */
typedef struct svdq_gemm_problem {
  const void* a16;     /* [M, K_pad] fp16 */
  const void* w16;     /* [N, K_pad] fp16 */
  const void* mid_hl;  /* [M, R2] bf16 (unused when R2 == 0) */
  const void* up_hl;   /* [N, R2] bf16 (unused when R2 == 0) */
  const void* bias;    /* [N] bf16, 16-byte aligned, or NULL */
  int epilogue;        /* enum svdq_epilogue */
  const void* aux;     /* epilogue operand [M, N] in out_dtype, row stride ld_aux */
  int64_t ld_aux;
  void* out;           /* [M, N], row stride ldo (multiple of 8) */
  int64_t ldo;
  int N;               /* multiple of 8 */
} svdq_gemm_problem;

/*
 * Up to four GEMMs that share M, K_pad and R2 (linears reading the same activations, such as a
 * transformer block's q / k / v projections) as one persistent launch: their 256x256 tiles are
 * numbered problem after problem and the CTA pairs walk them as one list, so a small problem
 * (few tiles) fills the waves of the others instead of leaving a ragged last wave of its own; the
 * split tail (workspace) applies to the group's last wave.  Each problem computes what
 * svdq_linear_gemm_epi computes for it.  num_problems in [1, 4]; every problem takes the same
 * epilogue operation (the kernel is compiled per operation); arguments as svdq_linear_gemm_epi.
 */
int svdq_linear_gemm_group(const svdq_gemm_problem* problems, int num_problems, int R2,
                           int out_dtype, int M, int K_pad,
                           void* workspace, size_t workspace_bytes, cudaStream_t stream);

/*
 * The launch plan of svdq_linear_gemm (with_workspace == 0) or
 * svdq_linear_gemm_ws (with_workspace != 0) for a shape on the current device:
 * out4 = {CTA pairs, tiles computed whole, K iterations per pair in the split
 * tail, tail iterations in total (0: no split)}.  A K iteration is 64 columns
 * of K_pad or of R2.  Host-only apart from the device attribute queries.
 */
int svdq_linear_gemm_schedule(int M, int N, int K_pad, int R2, int with_workspace, int* out4);

/*
 * The planner behind svdq_linear_gemm_schedule for a given number of 256x256
 * tiles, K iterations per tile and co-resident CTA pairs; same out4.  Host
 * only: makes no CUDA call.
 */
int svdq_linear_gemm_plan(int tiles, int iters, int max_pairs, int with_workspace, int* out4);

/*
 * Load-time preparation of the packed-weight GEMM's operands (replaces, like svdq_repack_weight,
 * the per-call unpack + dequantize of src/krea2_svdquant/quant/svd.py:128-135 and
 * quant/pack.py:26-70, but keeps the weight at half a byte per element):
 *   out_codes    [N, K_pad/2] u8: the checkpoint's codes (nibble q + 8, pack.py:47-56) with the
 *                nibbles of every 32-bit word reordered to [k0 k2 k4 k6 | k1 k3 k5 k7]
 *                (16-byte aligned);
 *   out_scales16 fp16, the group scales rounded to fp16 in tile order: for each 128-row tile t
 *                and each 256-k code group c, [128 rows][256 / w_group] contiguous at element
 *                ((t * ceil(K_pad / 256) + c) * 128 + row) * (256 / w_group); zero past N and K_pad
 *                (ceil(N / 128) * ceil(K_pad / 256) * 128 * (256 / w_group) elements, 16-byte aligned).
 * inexact (device int, may be NULL; not cleared here) is set to 1 when some scale or its
 * sixteenth is not an fp16 value; otherwise svdq_packed_gemm's weights equal svdq_repack_weight's
 * w16 bit for bit (bf16 scales in [2^-10, 8188], fp16 scales >= 2^-10, all group-scale zeros).
 *   w_group in {32, 64, 128, 256}, K_pad % w_group == 0, K_pad % 64 == 0; qweight 4-byte aligned.
 */
int svdq_prepare_packed(const void* qweight, const void* scales, int scale_dtype, int N, int K_pad,
                        int w_group, void* out_codes, void* out_scales16, int* inexact,
                        cudaStream_t stream);

/*
 * Packed-weight SVDQuant linear GEMM: the same computation as svdq_linear_gemm, with the weight
 * read as the half-byte codes + fp16 group scales of svdq_prepare_packed and converted on chip;
 * no fp16 weight is allocated.  Weight rows are the tcgen05 MMA's M dimension and tokens its N
 * (16 to 128 per tile), so small batches run small MMAs and read 4x fewer weight bytes.  Up to
 * 64 tokens the weights enter the MMA as exact fp16 integers q and each group's fp32 partial is
 * scaled by its weight scale in registers (as svdq_w4a4_gemm, with a16 for the activation);
 * above that they are converted to q * scale (exact, see above).  When the tiles leave SMs idle, a
 * cluster of 2, 4 or 8 CTAs splits K and sums its fp32 partials through distributed shared
 * memory in a fixed order (deterministic).  Replaces F.linear(x_hat, w_res) + F.linear(mid, l1)
 * + bias of svd.py:158-162 and the in-loop dequantization of kernels/triton/generic_int4.py:19-133.
 *   a16 [M, K_pad] fp16; K_pad % 64 == 0; w_group and the layouts of codes and scales16 as
 *   svdq_prepare_packed writes them; N % 8 == 0, ldo % 8 == 0;
 *   R2 % 64 == 0 (may be 0); out_dtype in {SVDQ_BF16, SVDQ_FP32}; bias may be NULL.
 */
int svdq_packed_gemm(const void* a16, const void* codes, const void* scales16, int w_group,
                     const void* mid_hl, const void* up_hl, int R2, const void* bias,
                     void* out, int out_dtype, int64_t ldo, int M, int N, int K_pad,
                     cudaStream_t stream);

/*
 * W4A4 GEMM on INT4 codes with kind::i8 tensor-core MMAs, for small batches: the weight read as
 * the half-byte codes + fp16 group scales of svdq_prepare_packed and converted to int8 on chip;
 * the activation as int8 codes with fp32 group scales (svdq_act_quant_i8).  Each K group's
 * products are summed exactly in int32 in tensor memory, then rescaled into fp32:
 *   out[m, n] = sum_g s_w[n, g] * s_a[m, g] * sum_{k in g} q_w[n, k] q_a[m, k]
 *             + mid_hl[m] . up_hl[n] + bias[n]
 * which is the reference's W4A4 formula (README.md:64; the residual product of
 * src/krea2_svdquant/quant/svd.py:158 on quantized activations, low-rank up + bias of
 * svd.py:159-162) with the int MMAs the reference's Blackwell kernel leaves as a TODO
 * (src/krea2_svdquant/kernels/gluon/blackwell_fused_svdquant.py:32-35).  Tokens are the MMA's N
 * dimension (16, 32 or 64 per tile), so the rescale costs a few instructions per output element
 * and group: meant for batches up to 64 tokens (larger M runs, in tiles of 64 tokens, but slower
 * than the fp16-operand GEMMs).  Split K over clusters as svdq_packed_gemm (deterministic).
 *   K_pad % 128 == 0; w_group in {64, 128, 256}, a_group in {64, 128}, both dividing K_pad;
 *   lda_s % 4 == 0 and lda_s >= M rounded up to 64 (entries past M are read, not used);
 *   codes8, ascales_t, codes, scales16 16-byte aligned; N % 8 == 0, ldo % 8 == 0;
 *   R2 % 64 == 0 (may be 0); out_dtype in {SVDQ_BF16, SVDQ_FP32}; bias may be NULL.
 */
int svdq_w4a4_gemm(const void* codes8, const float* ascales_t, int64_t lda_s, int a_group,
                   const void* codes, const void* scales16, int w_group,
                   const void* mid_hl, const void* up_hl, int R2, const void* bias,
                   void* out, int out_dtype, int64_t ldo, int M, int N, int K_pad,
                   cudaStream_t stream);

/*
 * svdq_w4a4_gemm for narrow batches (up to 16 tokens), with the products on mma.sync int8 fragments
 * in registers instead of tcgen05 and tensor memory: each warp streams the codes of 16 weight rows
 * by bulk asynchronous copies into a shared-memory ring of its own, turns each 32-bit word into the
 * u8 operand of one k-step with two mask operations, and rescales each K group's int32 result in
 * registers.  K is split over a cluster of two CTAs, whose fp32 partials are added through
 * distributed shared memory in a fixed order (deterministic).  The tcgen05 kernel spends these
 * batches converting codes into shared memory and reading each group's result back out of tensor
 * memory.  Same arguments, operand
 * layouts and result as svdq_w4a4_gemm (the fp32 sums in another order); also requires
 *   M <= 16, N % 128 == 0, K_pad % 512 == 0, a_group == w_group == 64, lda_s >= M;
 *   codes8, codes and scales16 16-byte aligned, ascales_t 4-byte aligned;
 *   R2 % 16 == 0 (may be 0), mid_hl / up_hl / bias 4-byte aligned; ldo even, out aligned to two
 *   elements.
 */
int svdq_w4a4_gemm_narrow(const void* codes8, const float* ascales_t, int64_t lda_s, int a_group,
                          const void* codes, const void* scales16, int w_group,
                          const void* mid_hl, const void* up_hl, int R2, const void* bias,
                          void* out, int out_dtype, int64_t ldo, int M, int N, int K_pad,
                          cudaStream_t stream);

/*
 * The launch plan of svdq_packed_gemm for a shape on the current device: out4 = {token tile TN,
 * CTAs per cluster along K, CTAs in the grid, CTAs per SM}.  Host only apart from device
 * attribute queries.
 */
int svdq_packed_gemm_plan(int M, int N, int K_pad, int* out4);

/*
 * Converter weight quantization on the GPU: an fp32 layer residual w [N, K]
 * (row stride ldw) -> packed INT4 codes [N, K_pad/2] (nibble q + 8, even k
 * low) and group scales [N, K_pad/group] as fp32, fp16 or bf16, with
 * K_pad = round_up(K, group).  Bit-exact with quantize_symmetric_int4 on fp32
 * input + pack_int4 (src/krea2_svdquant/quant/pack.py:6-23, 47-56) as
 * scripts/convert_simulated.py:197-203 calls them; fp16 / bf16 scales are the
 * fp32 scales rounded once.  group in {64, 128}; out_packed 4-byte aligned.
 */
int svdq_quantize_weight(const float* w, int64_t ldw, int N, int K, int group,
                         void* out_packed, void* out_scales, int scale_dtype, cudaStream_t stream);

/*
 * Block-weight prefetcher.  Replaces the synchronous per-tensor `.to(device)`
 * uploads of the reference's block offloader
 * (src/krea2_svdquant/runtime/block_offload.py:56-63, 157-173) with one
 * cudaMemcpyAsync per block from a pinned host arena into a device slot, on a
 * low-priority copy stream.  The caller owns the host arenas and the device
 * slots.  Per slot, an upload waits on the GPU for the slot's last release on
 * the compute stream; compute waits for the upload (and whatever the caller
 * enqueued after it on the copy stream) through svdq_prefetch_wait.
 *   create   -> copy stream + two events per slot (num_slots in [1, 64])
 *   begin    -> enqueue the upload of `bytes` from pinned host_src into dev_dst
 *   commit   -> mark the slot ready after everything on the copy stream so far
 *   wait     -> order `compute` after the slot's ready mark; timeout_ms >= 0 also
 *               blocks the host for at most timeout_ms (SVDQ_ERR_TIMEOUT after)
 *   release  -> record the end of the slot's use on `compute`
 *   sync     -> host wait (bounded by timeout_ms unless < 0) for all uploads
 */
typedef struct svdq_prefetcher svdq_prefetcher;
int svdq_prefetcher_create(int device, int num_slots, svdq_prefetcher** out);
int svdq_prefetcher_copy_stream(svdq_prefetcher* p, cudaStream_t* out);
int svdq_prefetch_begin(svdq_prefetcher* p, int slot, void* dev_dst, const void* host_src, size_t bytes);
int svdq_prefetch_commit(svdq_prefetcher* p, int slot);
int svdq_prefetch_wait(svdq_prefetcher* p, int slot, cudaStream_t compute, int timeout_ms);
int svdq_prefetch_release(svdq_prefetcher* p, int slot, cudaStream_t compute);
int svdq_prefetcher_sync(svdq_prefetcher* p, int timeout_ms);
int svdq_prefetcher_destroy(svdq_prefetcher* p);

#ifdef __cplusplus
}
#endif

#endif /* SVDQ_B200_H */
