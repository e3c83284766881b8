/*
 * scmp_b200.h -- C ABI of the B200 stochastic-computing (SC) matmul engine.
 *
 * Plain pointers and sizes only; every pointer is device memory on the
 * current CUDA device unless stated otherwise.  Every entry point returns
 * SCMP_OK (0) or a negative SCMP_E* code and never aborts; the message of the
 * last failure on the calling thread is available from scmp_last_error().
 *
 * The entry points replace the reference's kernel package `scmp_kernels`,
 * which the reference imports but does not vendor (.gitmodules:4-7):
 *   scmp_sc_matmul        <- scmp_kernels.sc.sc_matmul(a, b, granularity=,
 *                            mode=, sc_prec=, config=, group_a=, group_b=,
 *                            chunk_d=, stoc_len=)   as called at
 *                            sc_integration/sc_linear.py:137-147,170-180,
 *                            cls/sc_attention_patch.py:193-196,288-291,314-318,
 *                            det/sc_patch/sc_matmul.py:129-134,151-158,189-194
 *   row_stoc_len field    <- the per-level bucket loop of
 *                            sc_integration/sc_linear.py:255-265 and
 *                            cls/sc_attention_patch.py:217-240 (one launch
 *                            instead of one per level)
 *   slice_stoc_len field  <- the per-head bucket loop of
 *                            cls/sc_attention_patch.py:168-197
 *   k_segment field       <- 16 per-head launches on 16 streams of
 *                            sc_integration/head_aligned_comp.py:113-144
 *   scmp_sc_matmul_workspace_size: sizing helper (no reference counterpart;
 *                            the Triton package allocated internally)
 */
#ifndef SCMP_B200_H
#define SCMP_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SCMP_ABI_VERSION 1

#if defined(__GNUC__)
#define SCMP_API __attribute__((visibility("default")))
#else
#define SCMP_API
#endif

enum scmp_status {
  SCMP_OK = 0,
  SCMP_EINVAL = -1,       /* bad shape / argument */
  SCMP_ECUDA = -2,        /* a CUDA runtime call failed */
  SCMP_EWORKSPACE = -3,   /* workspace missing or too small */
  SCMP_EUNSUPPORTED = -4, /* valid request this library does not implement */
  SCMP_ETIMEOUT = -5      /* a bounded device-side wait gave up */
};

enum scmp_granularity { SCMP_PER_ROW = 0, SCMP_PER_HEAD = 1, SCMP_PER_TENSOR = 2 };
enum scmp_mode { SCMP_BIPOLAR = 0, SCMP_UNIPOLAR = 1 };
/* Element types of a, b and out (scmp_matmul_args.io_flags; 0 = all fp32). */
enum scmp_io_flags {
  SCMP_IO_A_BF16 = 1,   /* a is bf16: widened exactly to fp32 before quantisation */
  SCMP_IO_B_BF16 = 2,   /* b is bf16 */
  SCMP_IO_OUT_BF16 = 4, /* out is bf16: the fp32 result (bias included) rounded to nearest even */
  SCMP_IO_B_PACKED = 8, /* b is a buffer written by scmp_prepack_b for the same b arguments */
  SCMP_IO_A_QUANT = 16  /* a is a buffer written by scmp_softmax_quantize (per_row, group_a 1) */
};
enum scmp_engine {
  SCMP_ENGINE_AUTO = 0,
  SCMP_ENGINE_POPC = 1,    /* CUDA-core LOP3 + POPC over bit-packed streams */
  SCMP_ENGINE_TCGEN05 = 2  /* tcgen05 kind::i8 tensor-core bit-product GEMM */
};

typedef struct scmp_matmul_args {
  int32_t abi_version;      /* must be SCMP_ABI_VERSION */
  int32_t engine;           /* enum scmp_engine */
  /* a: [batch, M, K] contiguous; b: [batch_b, N, K] with batch_b in
   * {1, batch} (1 = b shared by every slice, e.g. a weight).  fp32, or bf16
   * per io_flags. */
  const void *a;
  const void *b;
  int64_t batch, batch_b, M, N, K;
  int32_t granularity;      /* enum scmp_granularity */
  int32_t mode;             /* enum scmp_mode */
  int32_t sc_prec;          /* p in [1, 8] (bipolar needs p >= 2) */
  int32_t stoc_len;         /* L in [1, 2^p]; used when no per-row table */
  int64_t group_a, group_b; /* per_row: rows per scale group (>= 1) */
  /* > 0: split K into K / k_segment segments (K % k_segment == 0, per_row
   * with group 1 only).  Each segment is quantised per row on its own and
   * rescaled on its own; the fp32 segment results are summed in segment
   * order, then the bias is added -- the head-aligned compensation of
   * sc_integration/head_aligned_comp.py:113-144 and the chunk-D summation of
   * sc_integration/sc_attention.py:337-376 in one launch.  0 = one segment. */
  int64_t k_segment;
  const uint8_t *pool;      /* stream pool R [pool_dims, 2^p] (uint8) */
  int32_t pool_dims;        /* reduction index d reads pool row d % pool_dims */
  int32_t io_flags;         /* enum scmp_io_flags bits; 0 = fp32 a, b, out */
  /* Optional per-a-row stream length [batch * M]: > 0 computes the row with
   * that L, 0 writes the pruned row (zeros + bias), < 0 leaves the output row
   * untouched (it belongs to another call).  NULL = every row uses stoc_len. */
  const int32_t *row_stoc_len;
  /* Optional per-slice stream length [batch] (same meaning, per slice). */
  const int32_t *slice_stoc_len;
  const float *bias;        /* nullable [N], added after the rescale */
  void *out;                /* [batch, M, N] fp32, or bf16 per io_flags */
  int32_t *acc_out;         /* nullable [batch, M, N] signed popcount sums */
  void *workspace;          /* device scratch, see scmp_sc_matmul_workspace_size */
  size_t workspace_bytes;
} scmp_matmul_args;

/* Size of the static scratch array behind scmp_sc_matmul_noalloc. */
#define SCMP_NOALLOC_SCRATCH_BYTES (32u * 1024u * 1024u)

/* Bytes of device scratch that scmp_sc_matmul needs for these arguments
 * (pointers may be NULL when only sizing).  Returns 0 on invalid arguments. */
SCMP_API size_t scmp_sc_matmul_workspace_size(const scmp_matmul_args *args);

/* SC estimate of a @ b^T per slice: quantise both operands, compare their
 * magnitudes against the pool (enable window for a, Sobol/LFSR stream for b),
 * accumulate signed popcounts, rescale to fp32.  Asynchronous on `stream`
 * (a cudaStream_t; NULL = legacy default stream). */
SCMP_API int scmp_sc_matmul(const scmp_matmul_args *args, void *stream);

/* scmp_sc_matmul for callers that cannot allocate device memory (no
 * reference counterpart).  A host binding the C ABI from plain C or an FFI
 * has no caching allocator, a cudaMalloc/cudaFree per call would synchronise
 * the device, and some runtimes reserve the whole memory budget up front; so
 * this variant ignores args->workspace and uses a fixed array compiled into
 * the library (SCMP_NOALLOC_SCRATCH_BYTES on every device that loads it, held
 * until exit).  It allocates nothing.  Problems needing more scratch than the
 * array holds (see scmp_sc_matmul_workspace_size) fail with SCMP_EWORKSPACE.
 * Every call on a device shares the array, which keeps the last call's
 * contents (the engine writes all scratch before reading it); calls whose
 * kernels overlap on the GPU race on it, so keep them on one stream.  The
 * first call on each device looks up the array's address with that device
 * current and caches it per (device, driver context): a host that makes
 * its own contexts (cuCtxCreate) gets the address in the context current at
 * the call.  Make the first call in each context before any stream capture
 * begins. */
SCMP_API int scmp_sc_matmul_noalloc(const scmp_matmul_args *args, void *stream);

/* Prepacked weights (no reference counterpart: the reference regenerates a
 * weight's stochastic streams in every call).  A weight b that stays fixed
 * across calls (batch_b = 1, no k_segment, 5 <= sc_prec <= 8, not unipolar
 * p = 8, pool_dims >= K) can be quantised and expanded into its tensor-core
 * operand bytes once; later calls pass the packed buffer as `b` with
 * SCMP_IO_B_PACKED and identical N, K, mode, granularity, group_b, sc_prec
 * and pool, and the engine loads those bytes with TMA instead of generating
 * them.  Results are bit-identical to passing b itself.  The buffer holds the
 * int16 codes, per-row scales and the operand bytes: e2m1 nibbles
 * [N][ceil8(K) * 2^p / 2] when sc_prec is 7 or 8 and N > 128 (loaded by the
 * e2m1 CTA pairs; 201 MB for a 3072 x 1024 weight at p = 7), else int8 bytes
 * [N][ceil8(K) * 2^p].
 * scmp_prepack_b_size returns its size (0 on invalid arguments; a, M and
 * the stream lengths are ignored); scmp_prepack_b writes it asynchronously on
 * `stream` (b fp32 or bf16 per io_flags). */
SCMP_API size_t scmp_prepack_b_size(const scmp_matmul_args *args);
SCMP_API int scmp_prepack_b(const scmp_matmul_args *args, void *packed, size_t packed_bytes,
                            void *stream);

/* Softmax fused into the Attn@V a operand.  Replaces, in one call, the
 * `attn.to(x.dtype) * self.scale` and `attn.softmax(dim=-1)` steps of
 * cls/sc_attention_patch.py:292-295 and the per-row quantisation that the
 * following sc_matmul(attn, v, granularity="per_row") applies to attn
 * (sc_integration/sc_linear.py:95-111).  For `rows` rows of K fp32 scores
 * (32 < K <= 1024), p = softmax(scale * scores) along each row with the
 * arithmetic of torch.softmax's fp32 kernel for such rows (the same bits),
 * then p quantised per row (mode, sc_prec) exactly as scmp_sc_matmul would
 * quantise it, into `a_quant`: int16 codes [rows][ceil8(K)], then per-row
 * scale, zero point and magnitude row sum, each region 256-byte aligned.
 * Pass that buffer as `a` of scmp_sc_matmul with SCMP_IO_A_QUANT, batch * M
 * = rows, the same K, mode and sc_prec, granularity per_row, group_a = 1:
 * the result is bit-identical to passing the probabilities, which never have
 * to be stored.  `probs` (nullable) receives them ([rows][K] fp32) anyway.
 * scmp_softmax_quantize_size returns the buffer's size (0 on bad sizes).
 * Asynchronous on `stream`; one launch. */
SCMP_API size_t scmp_softmax_quantize_size(int64_t rows, int64_t K);
SCMP_API int scmp_softmax_quantize(const float *scores, int64_t rows, int64_t K, float scale,
                                   int mode, int sc_prec, void *a_quant, size_t a_quant_bytes,
                                   float *probs, void *stream);

/* The fp32 elementwise steps of a transformer block around its matmuls,
 * fused (the block forward of the DINOv2 model the reference patches,
 * cls/sc_attention_patch.py:459-636: `x + ls1(attn(...))`, `fc2(act(fc1(...)))`,
 * `x + ls2(mlp(...))`, plus `block(x) + comp(x)` where a compensation is
 * installed).  Each step is rounded on its own in the order of the unfused
 * ops, so the results carry their bits.  Row-major [rows][cols] fp32;
 * asynchronous on `stream`; one launch each.
 * scmp_bias_gelu: y = gelu(y + bias) in place (exact GELU, erf form), for an
 * fc1 output computed without its bias.
 * scmp_scale_residual: out = (x + (y [+ bias]) * gamma) [+ extra]; bias and
 * extra nullable; out may alias x or y. */
SCMP_API int scmp_bias_gelu(float *y, const float *bias, int64_t rows, int64_t cols,
                            void *stream);
SCMP_API int scmp_scale_residual(float *out, const float *x, const float *y, const float *bias,
                                 const float *gamma, const float *extra, int64_t rows,
                                 int64_t cols, void *stream);

/* Split the fused qkv projection output of an attention block into the SC
 * matmul operands (the reshape / unbind / transpose of the qkv output in
 * cls/sc_attention_patch.py:248-328): qkv [B, N, 3, H, D] row-major ->
 * q, k [B, H, N, D] and vt [B, H, D, N] (v transposed), so that the per-head
 * Q@K^T and per-row Attn@V calls read contiguous slices.  Elements are
 * copied bit for bit (elem_bytes 2 for bf16 / fp16, 4 for fp32).  Requires
 * B * H <= 65535 and D <= 256.  Asynchronous on `stream`; two launches. */
SCMP_API int scmp_split_qkv(const void *qkv, int64_t B, int64_t N, int64_t H, int64_t D,
                            int elem_bytes, void *q, void *k, void *vt, void *stream);

/* Message of the last failure on this thread ("" if none). */
SCMP_API const char *scmp_last_error(void);

/* SCMP_ABI_VERSION of the loaded library. */
SCMP_API int scmp_abi_version(void);

/* Number of CUDA kernels this library has launched in this process (all
 * threads, all devices).  Instrumentation for launch accounting; no
 * reference counterpart. */
SCMP_API uint64_t scmp_kernel_launches(void);

/* Sticky device-side error flags of the current device, read synchronously
 * (bit 0: a bounded wait inside the tensor-core engine gave up, so some
 * output of an earlier call is invalid); reset != 0 clears them.  No
 * reference counterpart. */
SCMP_API int scmp_engine_status(int reset, unsigned int *flags);

/* Give-up path of the bounded device waits (test and instrumentation hooks;
 * no reference counterpart).  Every wait of the tensor-core engine on an
 * mbarrier spins for at most a limit, then marks its CTA aborted: the CTA
 * stops issuing work, waits for the tensor-core operations it already issued,
 * frees its tensor memory and returns, and the launch raises bit 0 of
 * scmp_engine_status.  scmp_debug_set_wait_limit sets that limit for later
 * launches on the current device (ns > 0; the default is 2 s).
 * scmp_debug_hold_producers(1) makes the operand producers of the e2m1
 * kernels (Lp = 128 / 256) first wait on a device flag that nothing sets, so
 * that every wait of those launches runs out (their outputs are not written);
 * scmp_debug_hold_producers(0) restores normal operation.  Both are
 * synchronous and apply to the current device only. */
SCMP_API int scmp_debug_set_wait_limit(uint64_t ns);
SCMP_API int scmp_debug_hold_producers(int on);

/* Roofline probe (synchronous; allocates a small scratch buffer): runs a
 * register-only loop of one instruction class on every SM of the current
 * device and returns its rate.  kind 0 = LOP3+POPC (bit-products/s),
 * 1 = mma.sync b1 AND.POPC (bit-products/s), 2 = mma.sync s8 (MACs/s),
 * 3 / 4 = tcgen05.mma kind::mxf4 M128 x N256 / N64 x K64 issued back to back
 * (MACs/s; one MAC of {-1, 0, +1} e2m1 operands is one SC bit-product).
 * Instrumentation only; no reference counterpart. */
SCMP_API int scmp_probe_int_peak(int kind, double *ops_per_second);

#ifdef __cplusplus
}
#endif

#endif /* SCMP_B200_H */
