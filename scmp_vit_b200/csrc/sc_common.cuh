// Shared definitions of the SC matmul engine (internal; the C ABI lives in
// include/scmp_b200.h).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "../../include/scmp_b200.h"

namespace scmp {

constexpr int kMaxPrec = 8;
constexpr int kMaxStream = 1 << kMaxPrec;  // 256

// One operand after quantisation: signed codes sigma*c (int16, [rows, K]) and
// per-row scale / zero point / magnitude row sum.
struct QuantPlane {
  const int16_t *code;
  const float *scale;
  const int32_t *zero;
  const int32_t *rowsum;
};

// Scale groups are contiguous row ranges: rows are split into slices of
// `slice_rows`, each slice into groups of `group_rows` (last one ragged).
struct GroupShape {
  int64_t rows;        // total rows
  int64_t slice_rows;  // rows per slice
  int64_t group_rows;  // rows per group (<= slice_rows)
  int64_t groups_per_slice;
  int64_t ngroups;
};

__host__ __device__ inline int64_t group_of_row(const GroupShape &g, int64_t r) {
  return (r / g.slice_rows) * g.groups_per_slice + (r % g.slice_rows) / g.group_rows;
}

// Everything a GEMM engine needs after quantisation.
struct GemmProblem {
  QuantPlane qa, qb;
  int64_t batch, batch_b, M, N, K;
  int64_t kseg;  // segment length (K when unsegmented); per-(row, segment) scales
  // code row stride: K rounded up to 8 (zero codes) when unsegmented, else K
  // (segment rows of kseg codes back to back)
  int64_t ldk;
  int nseg;      // K / kseg
  int mode, prec, stoc_len;
  const uint8_t *pool;  // [pool_dims, 2^prec]
  int pool_dims;
  const int32_t *row_L;    // nullable [batch*M]
  const int32_t *slice_L;  // nullable [batch]
  const float *bias;
  void *out;     // fp32, or bf16 when out_bf16
  int out_bf16;
  int32_t *acc_out;
  // stream table ST[pool_dims][2^p + 1][2^p / 32] (bit t of threshold v)
  const uint32_t *stream_table;
  // the thin strips' table SW[pool_dims][2^p + 1][2^p / 32 + 1]:
  // SW[d][v][w] = {ST[d][v][w] (0 at w = 2^p / 32), #{t < 32 w : R[d][t] < v}}
  const uint2 *strip_table;
  // pool complement PC[pool_dims][2^p] = 0x7F - (R >> shift) (tensor-core
  // row producers; shift = 1 for bipolar p = 8, else 0)
  const uint8_t *pool_comp;
  // prepacked b operand bytes (nullable; batch_b = 1): int8 [N][ldk * 2^p],
  // or with b_e2m1 e2m1 nibbles [N][ldk * 2^p / 2] (the e2m1 pair order)
  const uint8_t *b_streams;
  int b_e2m1;
  // window of (a row, b row) pairs per slice this launch computes
  int64_t m_lo, m_hi, n_lo, n_hi;
  // nullable int32 [ksplit, batch, M, N]: partial counts of K splits (the
  // workspace region sized by tc_ksplit; no split without it)
  int32_t *split_part;
};

// Per-row stream length in the engine's convention (see scmp_matmul_args).
__device__ __forceinline__ int row_stream_len(const GemmProblem &P, int64_t slice, int64_t grow) {
  if (P.row_L) return P.row_L[grow];
  if (P.slice_L) return P.slice_L[slice];
  return P.stoc_len;
}

// Store of one output element (fp32, or bf16 rounded to nearest even).
__device__ __forceinline__ void store_out(const GemmProblem &P, int64_t o, float y) {
  if (P.out_bf16)
    static_cast<__nv_bfloat16 *>(P.out)[o] = __float2bfloat16_rn(y);
  else
    static_cast<float *>(P.out)[o] = y;
}

// Rescale of one accumulator (bit-exact restatement of oracle/sc_oracle.c):
// F = 2^(2p) / (u L) depends on the row only, so epilogues compute it once per
// row (sc_rescale_factor) and apply it per element (sc_rescale_f).
__device__ __forceinline__ float sc_rescale_factor(int mode, int prec, int L) {
  return __fdiv_rn((float)(1u << (2 * prec)), (float)((mode == SCMP_BIPOLAR ? 4 : 1) * L));
}
__device__ __forceinline__ float sc_rescale_f(int mode, float F, int32_t acc, int64_t K, float sa,
                                              int32_t za, int32_t rsa, float sb, int32_t zb,
                                              int32_t rsb) {
  if (mode == SCMP_BIPOLAR) {
    const float fb = __fmul_rn(sb, F);
    return __fmul_rn(__fmul_rn((float)acc, sa), fb);
  }
  const long long corr = (long long)za * rsb + (long long)zb * rsa - K * (long long)za * (long long)zb;
  const float t = __fsub_rn(__fmul_rn((float)acc, F), __ll2float_rn(corr));
  return __fmul_rn(__fmul_rn(t, sa), sb);
}
__device__ __forceinline__ float sc_rescale(int mode, int prec, int L, int32_t acc, int64_t K,
                                            float sa, int32_t za, int32_t rsa, float sb,
                                            int32_t zb, int32_t rsb) {
  return sc_rescale_f(mode, sc_rescale_factor(mode, prec, L), acc, K, sa, za, rsa, sb, zb, rsb);
}

// Launchers (return cudaError_t of the launch).
// x is fp32, or bf16 when x_bf16 (widened exactly on load).
cudaError_t launch_row_stats(const void *x, bool x_bf16, int64_t rows, int64_t K, int mode,
                             float2 *stat, cudaStream_t s);
cudaError_t launch_group_stats(const float2 *stat, const GroupShape &g, int mode, int prec,
                               float *gscale, float *ginv, int32_t *gzero, cudaStream_t s);
cudaError_t launch_quantize(const void *x, bool x_bf16, const GroupShape &g, int64_t K,
                            int64_t ldc, int mode, int prec,
                            const float *gscale, const float *ginv, const int32_t *gzero,
                            int16_t *code, float *rscale, int32_t *rzero, int32_t *rsum,
                            cudaStream_t s);
// One-row scale groups: row stats, scale and codes in one launch (identical
// results to launch_row_stats + launch_group_stats + launch_quantize).
cudaError_t launch_quantize_rows(const void *x, bool x_bf16, int64_t rows, int64_t K,
                                 int64_t ldc, int mode, int prec, int16_t *code, float *rscale,
                                 int32_t *rzero, int32_t *rsum, cudaStream_t s);
// Whole-slice scale groups of short fp32 rows (per-head scaling of attention
// slices) in one launch, identical results to launch_row_stats +
// launch_group_stats + launch_quantize; false (nothing launched) when the
// shape does not qualify, else *err holds the launch status.
bool launch_quantize_slices(const float *x, const GroupShape &g, int64_t K, int64_t ldc,
                            int mode, int prec, int16_t *code, float *rscale, int32_t *rzero,
                            int32_t *rsum, cudaStream_t s, cudaError_t *err);
// Row softmax of scale * x (fp32, 32 < K <= 1024; torch.softmax's bits)
// and its per-row quantisation into codes [rows][ldc] and row records;
// probs (nullable) receives the probabilities.
cudaError_t launch_softmax_quantize(const float *x, int64_t rows, int K, float scale, int mode,
                                    int prec, int64_t ldc, int16_t *code, float *rscale,
                                    int32_t *rzero, int32_t *rsum, float *probs, cudaStream_t s);
// The stream table and, when strips != NULL, the thin strips' table (see
// GemmProblem::strip_table), from one pass over the pool.
cudaError_t launch_stream_table(const uint8_t *pool, int pool_dims, int prec, uint32_t *table,
                                uint2 *strips, cudaStream_t s);
// fp32 block glue (glue.cu): y = gelu(y + bias) in place; out = (x + (y [+
// bias]) * gamma) [+ extra], each step rounded on its own.
cudaError_t launch_bias_gelu(float *y, const float *bias, int64_t rows, int64_t cols,
                             cudaStream_t s);
cudaError_t launch_scale_residual(float *out, const float *x, const float *y, const float *bias,
                                  const float *gamma, const float *extra, int64_t rows,
                                  int64_t cols, cudaStream_t s);
// qkv [B, N, 3, H, D] -> q, k [B, H, N, D], vt [B, H, D, N] (elem_bytes 2 or 4)
cudaError_t launch_split_qkv(const void *qkv, int64_t B, int64_t N, int64_t H, int64_t D,
                             int elem_bytes, void *q, void *k, void *vt, cudaStream_t s);
// PC over max(pool_dims, rows) rows of 2^lp_log2 bytes (rows past the pool
// hold 0x7F).  nibble_pairs: each 8-byte group holds stream positions
// (0, 2, 4, 6, 1, 3, 5, 7) of its 8 (the e2m1 producers' order).
cudaError_t launch_pool_complement(const uint8_t *pool, int pool_dims, int64_t rows, int prec,
                                   int lp_log2, int shift, bool nibble_pairs, uint8_t *out,
                                   cudaStream_t s);
cudaError_t launch_gemm_popc(const GemmProblem &P, cudaStream_t s);
// b operand bytes of every row and k-block at Lp = 2^prec, as the row
// producers would generate them: out[n][k-block][128].  e2m1: nibbles in the
// e2m1 pair producers' order, 256 positions per 128 bytes (pool_comp is the
// natural-order complement either way).  pool_period > 0: reduction index d
// reads pool row d % pool_period (segmented K), else row d.
cudaError_t launch_pack_b_streams(const int16_t *code, int64_t N, int64_t ldk, int prec,
                                  int shift, bool e2m1, int64_t pool_period,
                                  const uint8_t *pool_comp, uint8_t *out, cudaStream_t s);
bool tc_supported(const GemmProblem &P);
int tc_block_n(int64_t N);
int tc_tile_n(const GemmProblem &P, int64_t N);
// true when the row-producer kernel runs this problem (it reads P.pool_comp)
bool tc_row_producers(const GemmProblem &P);
// log2 of the padded stream length Lp the tensor-core engine uses
int tc_stream_log2(const GemmProblem &P);
// true when launch_gemm_tc runs the e2m1 CTA-pair kernel on this window (its
// pool complement is laid out with nibble_pairs)
bool tc_nibble_pairs(const GemmProblem &P, int64_t m_rows, int64_t n_rows);
// *launches: kernels launched (the tile kernel, plus the reduce of K splits)
cudaError_t launch_gemm_tc(const GemmProblem &P, int64_t m_rows, int64_t n_rows,
                           unsigned int *error, cudaStream_t s, int *launches);
// K splits the tensor-core engine uses for this window (1 = none): problems
// whose e2m1 pair tiles would fill less than half of the SM pairs (e.g. one
// image's linear) split K so that every pair works; each split writes exact
// int32 partial counts and one reduce kernel rescales their sum.
int tc_ksplit(const GemmProblem &P, int64_t m_rows, int64_t n_rows);

// Message of the last failure on this thread (capi.cu).
void set_last_error(const char *msg);

// Driver context current on this thread (NULL if none or unknown).  A device
// symbol's address belongs to the context that loaded the module, so the
// per-device caches of symbol addresses are keyed by (ordinal, context): a
// host that makes its own contexts (cuCtxCreate) or resets a device gets its
// addresses looked up again instead of another context's.
void *current_context();

constexpr int kMaxCachedDevices = 64;
struct SymbolCache {
  void *ctx = nullptr;
  void *ptr = nullptr;
};

// Address of `symbol` in the current context, cached per device ordinal
// (looked up again when the current context differs from the cached one).
template <typename T>
cudaError_t cached_symbol_address(SymbolCache (&cache)[kMaxCachedDevices], std::mutex &mu,
                                  const T &symbol, void **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxCachedDevices) return cudaErrorInvalidDevice;
  void *ctx = current_context();
  std::lock_guard<std::mutex> lock(mu);
  SymbolCache &c = cache[dev];
  if (!c.ptr || c.ctx != ctx) {
    void *p = nullptr;
    if ((e = cudaGetSymbolAddress(&p, symbol)) != cudaSuccess) return e;
    if (!p) return cudaErrorInvalidSymbol;
    c.ptr = p;
    c.ctx = ctx;
  }
  *out = c.ptr;
  return cudaSuccess;
}
// Give-up path hooks of the tensor-core engine, on the current device
// (synchronous; SCMP_OK or an SCMP_E* code).
int debug_set_wait_limit(uint64_t ns);
int debug_hold_producers(int on);
// e2m1 MMA-rate probe (kind::mxf4, M = 128 x N = n x K = 64, n = 64 or 256):
// `blocks` CTAs each issue 4 * iters MMAs; bit 0 of *error = a wait gave up.
cudaError_t launch_probe_mma_mxf4(int n, int iters, int blocks, unsigned int *error,
                                  cudaStream_t s);

}  // namespace scmp
