// C ABI of the SC matmul engine (declared in include/scmp_b200.h).
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "sc_common.cuh"

namespace scmp {
namespace {

thread_local std::string g_last_error;
std::atomic<uint64_t> g_launches{0};

inline void count_launches(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

// Sticky device-side error word (bit 0: a bounded wait of the tensor-core
// engine gave up).  Read with scmp_engine_status.
__device__ unsigned int g_engine_error;
std::mutex g_err_mu;
SymbolCache g_err_ptr[kMaxCachedDevices];

unsigned int *engine_error_ptr() {
  void *p = nullptr;
  if (cached_symbol_address(g_err_ptr, g_err_mu, g_engine_error, &p) != cudaSuccess)
    return nullptr;
  return static_cast<unsigned int *>(p);
}

// Rows of the tail that the CUDA-core engine takes instead of padding a
// tensor-core tile (e.g. the 257th token).  Up to 8 rows run on the
// warp-per-output kernel at full occupancy; a longer tail costs less as a
// padded tensor-core tile (the tensor cores do ~5x the bit-products per
// second of the CUDA-core engine).
int64_t tc_rows(int64_t rows, int64_t tile) {
  const int64_t tail = rows % tile;
  if (tail != 0 && tail <= 8 && rows > tile) return rows - tail;
  return rows;
}

int fail(int code, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char *what) {
  return fail(SCMP_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

constexpr size_t kAlign = 256;
inline size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

struct OperandLayout {
  GroupShape g;
  int64_t ldc;  // code row stride
  size_t stat, gscale, ginv, gzero, code, rscale, rzero, rsum;  // offsets
};

// Bump allocator over the caller's workspace (or a null base when sizing).
struct Carver {
  size_t off = 0;
  size_t take(size_t bytes) {
    size_t at = off;
    off = align_up(off + bytes);
    return at;
  }
};

GroupShape make_groups(int gran, int64_t slices, int64_t rows_per_slice, int64_t group) {
  GroupShape g{};
  g.rows = slices * rows_per_slice;
  if (gran == SCMP_PER_TENSOR) {
    g.slice_rows = g.rows;
    g.group_rows = g.rows;
  } else if (gran == SCMP_PER_HEAD) {
    g.slice_rows = rows_per_slice;
    g.group_rows = rows_per_slice;
  } else {
    g.slice_rows = rows_per_slice;
    g.group_rows = group < rows_per_slice ? group : rows_per_slice;
  }
  g.groups_per_slice = (g.slice_rows + g.group_rows - 1) / g.group_rows;
  g.ngroups = (g.rows / g.slice_rows) * g.groups_per_slice;
  return g;
}

void layout_operand(Carver &c, OperandLayout &o, int64_t K, int64_t ldc) {
  o.ldc = ldc;
  const int64_t rows = o.g.rows, ng = o.g.ngroups;
  o.stat = c.take(sizeof(float2) * rows);
  o.gscale = c.take(sizeof(float) * ng);
  o.ginv = c.take(sizeof(float) * ng);
  o.gzero = c.take(sizeof(int32_t) * ng);
  o.code = c.take(sizeof(int16_t) * rows * ldc);
  o.rscale = c.take(sizeof(float) * rows);
  o.rzero = c.take(sizeof(int32_t) * rows);
  o.rsum = c.take(sizeof(int32_t) * rows);
}

struct Plan {
  OperandLayout A, B;
  size_t table = 0;
  size_t strips = 0;  // the thin strips' table (stream words with prefix counts)
  bool has_strips = false;  // carved only where the lane-group strip kernel can run
  size_t pool_comp = 0;
  int64_t pool_comp_rows = 0;
  int64_t ldk = 0;
  size_t split = 0;  // int32 [ksplit, batch, M, N] partial counts (ksplit > 1)
  int ksplit = 1;
  size_t total = 0;
};

int validate(const scmp_matmul_args *x) {
  if (!x) return fail(SCMP_EINVAL, "args is NULL");
  if (x->abi_version != SCMP_ABI_VERSION)
    return fail(SCMP_EINVAL, "abi_version %d != %d", x->abi_version, SCMP_ABI_VERSION);
  if (x->batch < 0 || x->M < 0 || x->N < 0 || x->K <= 0)
    return fail(SCMP_EINVAL, "bad shape batch=%lld M=%lld N=%lld K=%lld", (long long)x->batch,
                (long long)x->M, (long long)x->N, (long long)x->K);
  if (x->batch_b != 1 && x->batch_b != x->batch)
    return fail(SCMP_EINVAL, "batch_b=%lld must be 1 or batch=%lld", (long long)x->batch_b,
                (long long)x->batch);
  if (x->granularity < SCMP_PER_ROW || x->granularity > SCMP_PER_TENSOR)
    return fail(SCMP_EINVAL, "unknown granularity %d", x->granularity);
  if (x->mode != SCMP_BIPOLAR && x->mode != SCMP_UNIPOLAR)
    return fail(SCMP_EINVAL, "unknown mode %d", x->mode);
  if (x->sc_prec < 1 || x->sc_prec > kMaxPrec || (x->mode == SCMP_BIPOLAR && x->sc_prec < 2))
    return fail(SCMP_EINVAL, "sc_prec=%d out of range for mode %d", x->sc_prec, x->mode);
  const int T = 1 << x->sc_prec;
  if (!x->row_stoc_len && !x->slice_stoc_len && (x->stoc_len < 1 || x->stoc_len > T))
    return fail(SCMP_EINVAL, "stoc_len=%d must be in [1, 2^sc_prec=%d]", x->stoc_len, T);
  if (x->granularity == SCMP_PER_ROW && (x->group_a < 1 || x->group_b < 1))
    return fail(SCMP_EINVAL, "group_a/group_b must be >= 1");
  if (x->pool_dims <= 0) return fail(SCMP_EINVAL, "pool_dims must be positive");
  if (x->k_segment < 0) return fail(SCMP_EINVAL, "k_segment must be >= 0");
  if (x->k_segment > 0) {
    if (x->K % x->k_segment != 0)
      return fail(SCMP_EINVAL, "k_segment=%lld must divide K=%lld", (long long)x->k_segment,
                  (long long)x->K);
    if (x->k_segment != x->K &&
        (x->granularity != SCMP_PER_ROW || x->group_a != 1 || x->group_b != 1))
      return fail(SCMP_EINVAL, "k_segment needs granularity per_row with group_a=group_b=1");
  }
  if (x->io_flags & ~(SCMP_IO_A_BF16 | SCMP_IO_B_BF16 | SCMP_IO_OUT_BF16 | SCMP_IO_B_PACKED |
                      SCMP_IO_A_QUANT))
    return fail(SCMP_EINVAL, "unknown io_flags bits 0x%x", (unsigned)x->io_flags);
  if ((x->io_flags & SCMP_IO_A_QUANT) &&
      ((x->io_flags & SCMP_IO_A_BF16) || x->granularity != SCMP_PER_ROW || x->group_a != 1 ||
       (x->k_segment > 0 && x->k_segment != x->K)))
    return fail(SCMP_EINVAL,
                "a quantised a (SCMP_IO_A_QUANT) needs granularity per_row, group_a = 1 and "
                "no k_segment");
  if (x->engine != SCMP_ENGINE_AUTO && x->engine != SCMP_ENGINE_POPC &&
      x->engine != SCMP_ENGINE_TCGEN05)
    return fail(SCMP_EINVAL, "unknown engine %d", x->engine);
  return SCMP_OK;
}

int64_t seg_len(const scmp_matmul_args *x) { return x->k_segment > 0 ? x->k_segment : x->K; }

// A weight that can be prepacked: one b slice, a pool row per reduction index
// (per index inside its segment for segmented K), and 8-bit thresholds that
// fit the byte compare.  Segmented K packs e2m1 bytes for the e2m1 pairs only
// (sc_prec 7 or 8, segments of whole multiples of 8 indices).
int check_packable(const scmp_matmul_args *x) {
  if (x->batch_b != 1) return fail(SCMP_EINVAL, "prepacked b needs batch_b = 1");
  if (x->sc_prec < 5 || (x->mode == SCMP_UNIPOLAR && x->sc_prec == 8))
    return fail(SCMP_EUNSUPPORTED, "prepacked b needs 5 <= sc_prec <= 8 (not unipolar p = 8)");
  if (x->k_segment > 0 && x->k_segment != x->K) {
    if (x->sc_prec < 7 || (x->k_segment % 8) != 0)
      return fail(SCMP_EUNSUPPORTED,
                  "prepacked segmented b needs sc_prec 7 or 8 and k_segment a multiple of 8");
    if (x->pool_dims < x->k_segment)
      return fail(SCMP_EINVAL, "prepacked b needs pool_dims >= k_segment");
  } else if (x->pool_dims < x->K) {
    return fail(SCMP_EINVAL, "prepacked b needs pool_dims >= K");
  }
  const int64_t ldk = (x->K + 7) / 8 * 8;
  if ((ldk << x->sc_prec) >= ((int64_t)1 << 31))
    return fail(SCMP_EUNSUPPORTED, "prepacked b rows of %lld bytes are too long",
                (long long)(ldk << x->sc_prec));
  return SCMP_OK;
}

// Layout of a prepacked b buffer (offsets from its base): the b operand
// (group stats, int16 codes [N][ldk], per-row scale / zero / row sum), the
// pool complement at row stride 2^p, and the operand bytes: e2m1 nibbles
// [N][ldk * 2^p / 2] for the e2m1 CTA pairs (2^p = 128 or 256, N > 128, counts
// below 2^24), else int8 bytes [N][ldk * 2^p].
struct PackPlan {
  OperandLayout B;
  size_t pool_comp = 0, streams = 0, total = 0;
  int64_t ldk = 0, pool_rows = 0;
  bool e2m1 = false;
};

PackPlan make_pack_plan(const scmp_matmul_args *x) {
  PackPlan p;
  Carver c;
  const int64_t kseg = seg_len(x), nseg = x->K / kseg;
  if (nseg > 1) {
    // segment rows of kseg codes back to back ([N * nseg, kseg] = [N, K]),
    // one scale group per (row, segment); e2m1 bytes for the segmented pairs
    p.ldk = x->K;
    p.e2m1 = true;
    p.B.g = make_groups(SCMP_PER_ROW, 1, x->N * nseg, 1);
    layout_operand(c, p.B, kseg, kseg);
  } else {
    p.ldk = (x->K + 7) / 8 * 8;
    p.e2m1 = (x->sc_prec == 7 || x->sc_prec == 8) && x->N > 128 &&
             (p.ldk << x->sc_prec) < ((int64_t)1 << 24);
    p.B.g = make_groups(x->granularity, 1, x->N, x->group_b);
    layout_operand(c, p.B, x->K, p.ldk);
  }
  p.pool_rows = p.ldk > x->pool_dims ? p.ldk : x->pool_dims;
  p.pool_comp = c.take((size_t)p.pool_rows << x->sc_prec);
  p.streams = c.take((size_t)x->N * (size_t)(p.ldk << x->sc_prec) >> (p.e2m1 ? 1 : 0));
  p.total = c.off;
  return p;
}

// The fields of GemmProblem that the tensor-core routing reads, from the
// arguments alone (sizing precedes any pointer; the carved code planes are
// 256-byte aligned, as the routing requires).
GemmProblem routing_problem(const scmp_matmul_args *x, int64_t ldk) {
  GemmProblem P{};
  const int64_t kseg = seg_len(x);
  P.batch = x->batch;
  P.batch_b = x->batch_b;
  P.M = x->M;
  P.N = x->N;
  P.K = x->K;
  P.ldk = ldk;
  P.kseg = kseg;
  P.nseg = (int)(x->K / kseg);
  P.mode = x->mode;
  P.prec = x->sc_prec;
  P.stoc_len = x->stoc_len;
  P.pool_dims = x->pool_dims;
  static const int32_t marker = 0;
  P.row_L = x->row_stoc_len ? &marker : nullptr;
  P.slice_L = x->slice_stoc_len ? &marker : nullptr;
  P.acc_out = x->acc_out;
  if (x->io_flags & SCMP_IO_B_PACKED) {
    const PackPlan pk = make_pack_plan(x);
    static const uint8_t packed_marker = 0;
    P.b_streams = &packed_marker;
    P.b_e2m1 = pk.e2m1 ? 1 : 0;
  }
  return P;
}

// K splits the engine will use for these arguments (tensor-core route only).
int plan_ksplit(const scmp_matmul_args *x, int64_t ldk) {
  if (x->engine == SCMP_ENGINE_POPC || x->batch == 0 || x->M == 0 || x->N == 0) return 1;
  const GemmProblem P = routing_problem(x, ldk);
  if (!tc_supported(P)) return 1;
  return tc_ksplit(P, tc_rows(x->M, 256), tc_rows(x->N, tc_tile_n(P, x->N)));
}

Plan make_plan(const scmp_matmul_args *x) {
  Plan p;
  Carver c;
  // Segmented K is quantised as [rows * nseg, kseg] with one group per row.
  const int64_t kseg = seg_len(x), nseg = x->K / kseg;
  // a quantised a (SCMP_IO_A_QUANT) brings its own codes: no a planes here
  const bool a_quant = (x->io_flags & SCMP_IO_A_QUANT) != 0;
  p.A.g = make_groups(x->granularity, a_quant ? 0 : x->batch, x->M * nseg,
                      nseg > 1 ? 1 : x->group_a);
  p.B.g = make_groups(x->granularity, x->batch_b, x->N * nseg, nseg > 1 ? 1 : x->group_b);
  // unsegmented code rows are padded to a multiple of 8 (16-byte rows)
  const int64_t ldc = nseg > 1 ? kseg : (kseg + 7) / 8 * 8;
  p.ldk = nseg > 1 ? x->K : ldc;
  layout_operand(c, p.A, kseg, ldc);
  layout_operand(c, p.B, kseg, ldc);
  const int T = 1 << x->sc_prec;
  const int WT = T >= 32 ? T / 32 : 1;
  p.table = c.take(sizeof(uint32_t) * (size_t)x->pool_dims * (T + 1) * WT);
  // (the lane-group strip kernel takes unsegmented K <= 512; other strips
  // read the stream table alone)
  p.has_strips = x->K <= 512 && kseg == x->K;
  if (p.has_strips)
    p.strips = c.take(sizeof(uint2) * (size_t)x->pool_dims * (T + 1) * (WT + 1));
  p.pool_comp_rows = p.ldk > x->pool_dims ? p.ldk : x->pool_dims;
  p.pool_comp = c.take((size_t)p.pool_comp_rows * T);
  p.ksplit = plan_ksplit(x, p.ldk);
  if (p.ksplit > 1)
    p.split = c.take(sizeof(int32_t) * (size_t)p.ksplit * (size_t)(x->batch * x->M * x->N));
  p.total = c.off;
  return p;
}

// Layout of a quantised a operand (scmp_softmax_quantize, SCMP_IO_A_QUANT):
// int16 codes [rows][ldc] (ldc = K rounded up to 8, zero codes past K), then
// per-row scale (fp32), zero point and magnitude row sum (int32).
struct QuantALayout {
  size_t code = 0, rscale = 0, rzero = 0, rsum = 0, total = 0;
  int64_t ldc = 0;
};
QuantALayout quant_a_layout(int64_t rows, int64_t K) {
  QuantALayout q;
  Carver c;
  q.ldc = (K + 7) / 8 * 8;
  q.code = c.take(sizeof(int16_t) * (size_t)rows * (size_t)q.ldc);
  q.rscale = c.take(sizeof(float) * (size_t)rows);
  q.rzero = c.take(sizeof(int32_t) * (size_t)rows);
  q.rsum = c.take(sizeof(int32_t) * (size_t)rows);
  q.total = c.off;
  return q;
}

int quantize_operand(const void *x, bool x_bf16, const OperandLayout &o, int64_t K, int mode,
                     int prec, unsigned char *ws, cudaStream_t s) {
  cudaError_t e;
  auto *stat = reinterpret_cast<float2 *>(ws + o.stat);
  auto *gscale = reinterpret_cast<float *>(ws + o.gscale);
  auto *ginv = reinterpret_cast<float *>(ws + o.ginv);
  auto *gzero = reinterpret_cast<int32_t *>(ws + o.gzero);
  if (o.g.group_rows == 1) {
    // one row per scale group: stats, scale and codes in one launch
    if ((e = launch_quantize_rows(x, x_bf16, o.g.rows, K, o.ldc, mode, prec,
                                  reinterpret_cast<int16_t *>(ws + o.code),
                                  reinterpret_cast<float *>(ws + o.rscale),
                                  reinterpret_cast<int32_t *>(ws + o.rzero),
                                  reinterpret_cast<int32_t *>(ws + o.rsum), s)) != cudaSuccess)
      return cuda_fail(e, "quantize_rows launch");
    if (o.g.rows > 0) count_launches(1);
    return SCMP_OK;
  }
  if (!x_bf16 &&
      launch_quantize_slices(static_cast<const float *>(x), o.g, K, o.ldc, mode, prec,
                             reinterpret_cast<int16_t *>(ws + o.code),
                             reinterpret_cast<float *>(ws + o.rscale),
                             reinterpret_cast<int32_t *>(ws + o.rzero),
                             reinterpret_cast<int32_t *>(ws + o.rsum), s, &e)) {
    if (e != cudaSuccess) return cuda_fail(e, "quantize_slices launch");
    if (o.g.rows > 0) count_launches(1);
    return SCMP_OK;
  }
  if ((e = launch_row_stats(x, x_bf16, o.g.rows, K, mode, stat, s)) != cudaSuccess)
    return cuda_fail(e, "row_stats launch");
  if ((e = launch_group_stats(stat, o.g, mode, prec, gscale, ginv, gzero, s)) != cudaSuccess)
    return cuda_fail(e, "group_stats launch");
  if ((e = launch_quantize(x, x_bf16, o.g, K, o.ldc, mode, prec, gscale, ginv, gzero,
                           reinterpret_cast<int16_t *>(ws + o.code),
                           reinterpret_cast<float *>(ws + o.rscale),
                           reinterpret_cast<int32_t *>(ws + o.rzero),
                           reinterpret_cast<int32_t *>(ws + o.rsum), s)) != cudaSuccess)
    return cuda_fail(e, "quantize launch");
  if (o.g.rows > 0) count_launches(3);
  return SCMP_OK;
}

QuantPlane plane_of(const OperandLayout &o, unsigned char *ws) {
  QuantPlane q;
  q.code = reinterpret_cast<const int16_t *>(ws + o.code);
  q.scale = reinterpret_cast<const float *>(ws + o.rscale);
  q.zero = reinterpret_cast<const int32_t *>(ws + o.rzero);
  q.rowsum = reinterpret_cast<const int32_t *>(ws + o.rsum);
  return q;
}

}  // namespace

void set_last_error(const char *msg) { g_last_error = msg ? msg : ""; }

void *current_context() {
  using GetCurrent = int (*)(void **);
  static std::once_flag once;
  static GetCurrent fn = nullptr;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetCurrent>(p);
  });
  void *ctx = nullptr;
  if (fn && fn(&ctx) != 0) ctx = nullptr;
  return ctx;
}

}  // namespace scmp

using namespace scmp;

extern "C" {

const char *scmp_last_error(void) { return g_last_error.c_str(); }

int scmp_abi_version(void) { return SCMP_ABI_VERSION; }

uint64_t scmp_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

int scmp_engine_status(int reset, unsigned int *flags) {
  if (!flags) return fail(SCMP_EINVAL, "flags is NULL");
  cudaError_t e = cudaMemcpyFromSymbol(flags, g_engine_error, sizeof(unsigned int));
  if (e != cudaSuccess) return cuda_fail(e, "reading the engine error word");
  if (reset) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_engine_error, &zero, sizeof(unsigned int));
    if (e != cudaSuccess) return cuda_fail(e, "clearing the engine error word");
  }
  return SCMP_OK;
}

int scmp_debug_set_wait_limit(uint64_t ns) {
  g_last_error.clear();
  return debug_set_wait_limit(ns);
}

int scmp_debug_hold_producers(int on) {
  g_last_error.clear();
  return debug_hold_producers(on);
}

size_t scmp_prepack_b_size(const scmp_matmul_args *args) {
  if (validate(args) != SCMP_OK || check_packable(args) != SCMP_OK) return 0;
  if (args->N == 0) return kAlign;
  return make_pack_plan(args).total;
}

int scmp_prepack_b(const scmp_matmul_args *args, void *packed, size_t packed_bytes,
                   void *stream) {
  g_last_error.clear();
  int rc = validate(args);
  if (rc != SCMP_OK) return rc;
  if ((rc = check_packable(args)) != SCMP_OK) return rc;
  const scmp_matmul_args &x = *args;
  if (x.io_flags & SCMP_IO_B_PACKED) return fail(SCMP_EINVAL, "b is already packed");
  if (x.N == 0) return SCMP_OK;
  if (!x.b || !x.pool || !packed) return fail(SCMP_EINVAL, "b, pool and packed must be non-NULL");
  const PackPlan pk = make_pack_plan(&x);
  if (packed_bytes < pk.total)
    return fail(SCMP_EWORKSPACE, "packed buffer needs %zu bytes, got %zu", pk.total,
                packed_bytes);
  if ((reinterpret_cast<uintptr_t>(packed) & (kAlign - 1)) != 0)
    return fail(SCMP_EINVAL, "packed buffer must be %zu-byte aligned", kAlign);
  auto *pb = static_cast<unsigned char *>(packed);
  auto s = static_cast<cudaStream_t>(stream);
  const int64_t kseg = seg_len(&x);
  if ((rc = quantize_operand(x.b, (x.io_flags & SCMP_IO_B_BF16) != 0, pk.B, kseg, x.mode,
                             x.sc_prec, pb, s)) != SCMP_OK)
    return rc;
  const int shift = (x.mode == SCMP_BIPOLAR && x.sc_prec == 8) ? 1 : 0;
  cudaError_t e;
  if ((e = launch_pool_complement(x.pool, x.pool_dims, pk.pool_rows, x.sc_prec, x.sc_prec, shift,
                                  false, pb + pk.pool_comp, s)) != cudaSuccess)
    return cuda_fail(e, "pool_complement launch");
  if ((e = launch_pack_b_streams(reinterpret_cast<const int16_t *>(pb + pk.B.code), x.N, pk.ldk,
                                 x.sc_prec, shift, pk.e2m1, kseg < x.K ? kseg : 0,
                                 pb + pk.pool_comp, pb + pk.streams, s)) != cudaSuccess)
    return cuda_fail(e, "pack_b_streams launch");
  count_launches(2);
  return SCMP_OK;
}

int scmp_split_qkv(const void *qkv, int64_t B, int64_t N, int64_t H, int64_t D, int elem_bytes,
                   void *q, void *k, void *vt, void *stream) {
  g_last_error.clear();
  if (B < 0 || N < 0 || H < 0 || D < 0) return fail(SCMP_EINVAL, "negative size");
  if (elem_bytes != 2 && elem_bytes != 4)
    return fail(SCMP_EINVAL, "elem_bytes must be 2 or 4, got %d", elem_bytes);
  if (B * H > 65535 || D > 256)
    return fail(SCMP_EUNSUPPORTED, "split_qkv supports B * H <= 65535 and D <= 256");
  if (B == 0 || N == 0 || H == 0 || D == 0) return SCMP_OK;
  if (!qkv || !q || !k || !vt) return fail(SCMP_EINVAL, "qkv, q, k and vt must be non-NULL");
  const cudaError_t e =
      launch_split_qkv(qkv, B, N, H, D, elem_bytes, q, k, vt, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "split_qkv launch");
  count_launches(2);
  return SCMP_OK;
}

int scmp_bias_gelu(float *y, const float *bias, int64_t rows, int64_t cols, void *stream) {
  g_last_error.clear();
  if (rows < 0 || cols < 0) return fail(SCMP_EINVAL, "negative size");
  if (rows == 0 || cols == 0) return SCMP_OK;
  if (!y || !bias) return fail(SCMP_EINVAL, "y and bias must be non-NULL");
  const cudaError_t e = launch_bias_gelu(y, bias, rows, cols, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "bias_gelu launch");
  count_launches(1);
  return SCMP_OK;
}

int scmp_scale_residual(float *out, const float *x, const float *y, const float *bias,
                        const float *gamma, const float *extra, int64_t rows, int64_t cols,
                        void *stream) {
  g_last_error.clear();
  if (rows < 0 || cols < 0) return fail(SCMP_EINVAL, "negative size");
  if (rows == 0 || cols == 0) return SCMP_OK;
  if (!out || !x || !y || !gamma) return fail(SCMP_EINVAL, "out, x, y and gamma must be non-NULL");
  const cudaError_t e = launch_scale_residual(out, x, y, bias, gamma, extra, rows, cols,
                                              static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "scale_residual launch");
  count_launches(1);
  return SCMP_OK;
}

size_t scmp_softmax_quantize_size(int64_t rows, int64_t K) {
  if (rows < 0 || K <= 0) return 0;
  return quant_a_layout(rows, K).total;
}

int scmp_softmax_quantize(const float *scores, int64_t rows, int64_t K, float scale, int mode,
                          int sc_prec, void *a_quant, size_t a_quant_bytes, float *probs,
                          void *stream) {
  g_last_error.clear();
  if (rows < 0 || K <= 0)
    return fail(SCMP_EINVAL, "bad shape rows=%lld K=%lld", (long long)rows, (long long)K);
  if (K <= 32 || K > 1024)
    return fail(SCMP_EUNSUPPORTED, "softmax_quantize takes rows of 33 to 1024 values, got %lld",
                (long long)K);
  if (mode != SCMP_BIPOLAR && mode != SCMP_UNIPOLAR)
    return fail(SCMP_EINVAL, "unknown mode %d", mode);
  if (sc_prec < 1 || sc_prec > kMaxPrec || (mode == SCMP_BIPOLAR && sc_prec < 2))
    return fail(SCMP_EINVAL, "sc_prec=%d out of range for mode %d", sc_prec, mode);
  const QuantALayout q = quant_a_layout(rows, K);
  if (rows == 0) return SCMP_OK;
  if (!scores || !a_quant) return fail(SCMP_EINVAL, "scores and a_quant must be non-NULL");
  if (a_quant_bytes < q.total)
    return fail(SCMP_EWORKSPACE, "a_quant needs %zu bytes, got %zu", q.total, a_quant_bytes);
  if ((reinterpret_cast<uintptr_t>(a_quant) & (kAlign - 1)) != 0)
    return fail(SCMP_EINVAL, "a_quant must be %zu-byte aligned", kAlign);
  auto *pa = static_cast<unsigned char *>(a_quant);
  const cudaError_t e = launch_softmax_quantize(
      scores, rows, (int)K, scale, mode, sc_prec, q.ldc, reinterpret_cast<int16_t *>(pa + q.code),
      reinterpret_cast<float *>(pa + q.rscale), reinterpret_cast<int32_t *>(pa + q.rzero),
      reinterpret_cast<int32_t *>(pa + q.rsum), probs, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "softmax_quantize launch");
  count_launches(1);
  return SCMP_OK;
}

size_t scmp_sc_matmul_workspace_size(const scmp_matmul_args *args) {
  if (validate(args) != SCMP_OK) return 0;
  if (args->batch == 0 || args->M == 0 || args->N == 0) return kAlign;
  return make_plan(args).total;
}

int scmp_sc_matmul(const scmp_matmul_args *args, void *stream) {
  g_last_error.clear();
  int rc = validate(args);
  if (rc != SCMP_OK) return rc;
  const scmp_matmul_args &x = *args;
  if (x.batch == 0 || x.M == 0 || x.N == 0) return SCMP_OK;
  if (!x.a || !x.b || !x.pool || !x.out)
    return fail(SCMP_EINVAL, "a, b, pool and out must be non-NULL");
  const Plan plan = make_plan(&x);
  if (!x.workspace || x.workspace_bytes < plan.total)
    return fail(SCMP_EWORKSPACE, "workspace needs %zu bytes, got %zu", plan.total,
                x.workspace ? x.workspace_bytes : (size_t)0);
  auto *ws = static_cast<unsigned char *>(x.workspace);
  auto s = static_cast<cudaStream_t>(stream);

  const int64_t kseg = seg_len(&x);
  const bool packed = (x.io_flags & SCMP_IO_B_PACKED) != 0;
  const bool a_quant = (x.io_flags & SCMP_IO_A_QUANT) != 0;
  if (packed && (rc = check_packable(&x)) != SCMP_OK) return rc;
  if (!a_quant && (rc = quantize_operand(x.a, (x.io_flags & SCMP_IO_A_BF16) != 0, plan.A, kseg,
                                         x.mode, x.sc_prec, ws, s)) != SCMP_OK)
    return rc;
  if (!packed && (rc = quantize_operand(x.b, (x.io_flags & SCMP_IO_B_BF16) != 0, plan.B, kseg,
                                        x.mode, x.sc_prec, ws, s)) != SCMP_OK)
    return rc;
  auto *table = reinterpret_cast<uint32_t *>(ws + plan.table);
  cudaError_t e;

  GemmProblem P{};
  if (a_quant) {
    // codes and row records written by scmp_softmax_quantize for these rows
    const QuantALayout qa = quant_a_layout(x.batch * x.M, x.K);
    auto *pa = static_cast<unsigned char *>(const_cast<void *>(x.a));
    P.qa.code = reinterpret_cast<const int16_t *>(pa + qa.code);
    P.qa.scale = reinterpret_cast<const float *>(pa + qa.rscale);
    P.qa.zero = reinterpret_cast<const int32_t *>(pa + qa.rzero);
    P.qa.rowsum = reinterpret_cast<const int32_t *>(pa + qa.rsum);
  } else {
    P.qa = plane_of(plan.A, ws);
  }
  if (packed) {
    // b's codes, scales and operand bytes were written by scmp_prepack_b
    const PackPlan pk = make_pack_plan(&x);
    auto *pb = static_cast<unsigned char *>(const_cast<void *>(x.b));
    P.qb = plane_of(pk.B, pb);
    P.b_streams = pb + pk.streams;
    P.b_e2m1 = pk.e2m1 ? 1 : 0;
  } else {
    P.qb = plane_of(plan.B, ws);
  }
  P.batch = x.batch;
  P.batch_b = x.batch_b;
  P.M = x.M;
  P.N = x.N;
  P.K = x.K;
  P.ldk = plan.ldk;
  P.kseg = kseg;
  P.nseg = (int)(x.K / kseg);
  P.mode = x.mode;
  P.prec = x.sc_prec;
  P.stoc_len = x.stoc_len;
  P.pool = x.pool;
  P.pool_dims = x.pool_dims;
  P.row_L = x.row_stoc_len;
  P.slice_L = x.slice_stoc_len;
  P.bias = x.bias;
  P.out = x.out;
  P.out_bf16 = (x.io_flags & SCMP_IO_OUT_BF16) != 0;
  P.acc_out = x.acc_out;
  P.stream_table = table;
  P.strip_table = plan.has_strips ? reinterpret_cast<const uint2 *>(ws + plan.strips) : nullptr;
  P.pool_comp = ws + plan.pool_comp;
  P.m_lo = 0;
  P.m_hi = x.M;
  P.n_lo = 0;
  P.n_hi = x.N;
  P.split_part = plan.ksplit > 1 ? reinterpret_cast<int32_t *>(ws + plan.split) : nullptr;

  bool use_tc = false;
  if (x.engine == SCMP_ENGINE_TCGEN05) {
    if (!tc_supported(P))
      return fail(SCMP_EUNSUPPORTED,
                  "tcgen05 engine needs 5 <= sc_prec <= 8, one K segment, and not unipolar at p=8");
    use_tc = true;
  } else if (x.engine == SCMP_ENGINE_AUTO) {
    use_tc = tc_supported(P);
  }
  int64_t m_tc = 0, n_tc = 0;
  if (use_tc) {
    unsigned int *err = engine_error_ptr();
    if (!err) return fail(SCMP_ECUDA, "cannot resolve the engine error word");
    m_tc = tc_rows(x.M, 256);
    n_tc = tc_rows(x.N, tc_tile_n(P, x.N));
    if (tc_row_producers(P)) {
      const int shift = (x.mode == SCMP_BIPOLAR && x.sc_prec == 8) ? 1 : 0;
      if ((e = launch_pool_complement(x.pool, x.pool_dims, plan.pool_comp_rows, x.sc_prec,
                                      tc_stream_log2(P), shift, tc_nibble_pairs(P, m_tc, n_tc),
                                      ws + plan.pool_comp, s)) !=
          cudaSuccess)
        return cuda_fail(e, "pool_complement launch");
      count_launches(1);
    }
    int launched = 0;
    if ((e = launch_gemm_tc(P, m_tc, n_tc, err, s, &launched)) != cudaSuccess)
      return cuda_fail(e, "gemm_tc launch");
    count_launches((uint64_t)launched);
  }
  // CUDA-core engine: everything (no tensor-core path) or the ragged strips
  // the tensor-core tiles leave (rows >= m_tc; columns >= n_tc of rows < m_tc).
  const bool strip_m = use_tc && m_tc < x.M;
  const bool strip_n = use_tc && n_tc < x.N && m_tc > 0;
  if (!use_tc || strip_m || strip_n) {
    if ((e = launch_stream_table(x.pool, x.pool_dims, x.sc_prec, table,
                                 plan.has_strips ? reinterpret_cast<uint2 *>(ws + plan.strips)
                                                 : nullptr,
                                 s)) !=
        cudaSuccess)
      return cuda_fail(e, "stream_table launch");
    count_launches(1);
  }
  if (!use_tc) {
    if ((e = launch_gemm_popc(P, s)) != cudaSuccess) return cuda_fail(e, "gemm_popc launch");
    count_launches(1);
  }
  if (strip_m) {
    GemmProblem Q = P;
    Q.m_lo = m_tc;
    if ((e = launch_gemm_popc(Q, s)) != cudaSuccess) return cuda_fail(e, "gemm_popc launch");
    count_launches(1);
  }
  if (strip_n) {
    GemmProblem Q = P;
    Q.m_hi = m_tc;
    Q.n_lo = n_tc;
    if ((e = launch_gemm_popc(Q, s)) != cudaSuccess) return cuda_fail(e, "gemm_popc launch");
    count_launches(1);
  }
  return SCMP_OK;
}

}  // extern "C"
