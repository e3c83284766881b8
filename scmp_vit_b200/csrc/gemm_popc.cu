// SC GEMM on CUDA cores: LOP3 + POPC over bit-packed streams.
//
// For every (m, n, d) the enable window of a (a prefix mask of k bits) is
// ANDed with the Sobol/LFSR stream of b (bit t = [R[d][t] < c_b]) and the
// popcount is accumulated with the sign product.  This is the integer-pipe
// formulation of the SC inner product; it is kept as the baseline engine and
// as the engine for shapes the tensor-core path does not take.
#include "sc_common.cuh"

namespace scmp {
namespace {

constexpr int BM = 64;
constexpr int BN = 64;
constexpr int kThreads = 256;

template <int LW>
struct PopcCfg {
  static constexpr int BD = LW >= 8 ? 8 : 16;  // reduction dims per stage
  static constexpr size_t smem_bytes =
      (size_t)BD * (BM + BN) * LW * sizeof(uint32_t) + (size_t)BD * (BM + BN);
};

template <int LW>
__global__ void __launch_bounds__(kThreads) gemm_popc_kernel(GemmProblem P) {
  using Cfg = PopcCfg<LW>;
  constexpr int BD = Cfg::BD;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint32_t *sA = reinterpret_cast<uint32_t *>(smem_raw);  // [BD][BM][LW]
  uint32_t *sB = sA + BD * BM * LW;                        // [BD][BN][LW]
  int8_t *gA = reinterpret_cast<int8_t *>(sB + BD * BN * LW);  // [BD][BM]
  int8_t *gB = gA + BD * BM;                                    // [BD][BN]

  const int64_t slice = blockIdx.z;
  const int64_t slice_b = P.batch_b == 1 ? 0 : slice;
  const int64_t m0 = P.m_lo + (int64_t)blockIdx.y * BM;
  const int64_t n0 = P.n_lo + (int64_t)blockIdx.x * BN;
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int T = 1 << P.prec;
  const int WT = T >= 32 ? T / 32 : 1;

  int32_t acc[4][4], acc_sum[4][4];
  float y[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) { acc[i][j] = 0; acc_sum[i][j] = 0; y[i][j] = 0.0f; }

  for (int64_t d0 = 0; d0 < P.K; d0 += BD) {
    // ---- stage A: enable windows (prefix masks) and signs
    for (int idx = tid; idx < BM * BD; idx += kThreads) {
      const int m = idx / BD, dd = idx % BD;
      const int64_t gm = m0 + m, d = d0 + dd;
      int k = 0, s = 1;
      if (gm < P.m_hi && d < P.K) {
        const int64_t grow = slice * P.M + gm;
        const int L = row_stream_len(P, slice, grow);
        const int c = P.qa.code[grow * P.ldk + d];
        s = c < 0 ? -1 : 1;
        if (L > 0) k = ((c < 0 ? -c : c) * L) >> P.prec;
      }
      uint32_t *dst = sA + (dd * BM + m) * LW;
#pragma unroll
      for (int w = 0; w < LW; ++w) {
        const int lo = 32 * w;
        dst[w] = k >= lo + 32 ? 0xffffffffu : (k > lo ? ((1u << (k - lo)) - 1u) : 0u);
      }
      gA[dd * BM + m] = (int8_t)s;
    }
    // ---- stage B: streams from the table, and signs
    for (int idx = tid; idx < BN * BD; idx += kThreads) {
      const int n = idx / BD, dd = idx % BD;
      const int64_t gn = n0 + n, d = d0 + dd;
      uint32_t *dst = sB + (dd * BN + n) * LW;
      int s = 1;
      if (gn < P.n_hi && d < P.K) {
        const int c = P.qb.code[(slice_b * P.N + gn) * P.ldk + d];
        s = c < 0 ? -1 : 1;
        const int v = c < 0 ? -c : c;
        const uint32_t *st =
            P.stream_table + ((int64_t)(d % P.pool_dims) * (T + 1) + v) * WT;
#pragma unroll
        for (int w = 0; w < LW; ++w) dst[w] = st[w];
      } else {
#pragma unroll
        for (int w = 0; w < LW; ++w) dst[w] = 0u;
      }
      gB[dd * BN + n] = (int8_t)s;
    }
    __syncthreads();
    // ---- popcount inner product
    for (int dd = 0; dd < BD; ++dd) {
      uint32_t a[4][LW], b[4][LW];
      int sa[4], sb[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t *pa = sA + (dd * BM + ty + 16 * i) * LW;
        const uint32_t *pb = sB + (dd * BN + tx + 16 * i) * LW;
#pragma unroll
        for (int w = 0; w < LW; ++w) { a[i][w] = pa[w]; b[i][w] = pb[w]; }
        sa[i] = gA[dd * BM + ty + 16 * i];
        sb[i] = gB[dd * BN + tx + 16 * i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          int cnt = 0;
#pragma unroll
          for (int w = 0; w < LW; ++w) cnt += __popc(a[i][w] & b[j][w]);
          acc[i][j] += (sa[i] * sb[j]) * cnt;
        }
      // ---- end of a segment: rescale it and add it to the fp32 sum
      const int64_t d = d0 + dd;
      if (d < P.K && (d + 1) % P.kseg == 0) {
        const int64_t seg = d / P.kseg;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int64_t gm = m0 + ty + 16 * i;
          if (gm >= P.m_hi) continue;
          const int64_t grow = slice * P.M + gm;
          const int L = row_stream_len(P, slice, grow);
          const int64_t ra = grow * P.nseg + seg;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int64_t gn = n0 + tx + 16 * j;
            if (gn < P.n_hi && L > 0) {
              const int64_t rb = (slice_b * P.N + gn) * P.nseg + seg;
              const float r = sc_rescale(P.mode, P.prec, L, acc[i][j], P.kseg, P.qa.scale[ra],
                                         P.qa.zero[ra], P.qa.rowsum[ra], P.qb.scale[rb],
                                         P.qb.zero[rb], P.qb.rowsum[rb]);
              y[i][j] = seg == 0 ? r : __fadd_rn(y[i][j], r);
              acc_sum[i][j] += acc[i][j];
            }
            acc[i][j] = 0;
          }
        }
      }
    }
    __syncthreads();
  }

  // ---- epilogue: bias, store
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t gm = m0 + ty + 16 * i;
    if (gm >= P.m_hi) continue;
    const int64_t grow = slice * P.M + gm;
    const int L = row_stream_len(P, slice, grow);
    if (L < 0) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t gn = n0 + tx + 16 * j;
      if (gn >= P.n_hi) continue;
      float v = L > 0 ? y[i][j] : 0.0f;
      if (P.bias) v = __fadd_rn(v, P.bias[gn]);
      const int64_t o = grow * P.N + gn;
      store_out(P, o, v);
      if (P.acc_out) P.acc_out[o] = L > 0 ? acc_sum[i][j] : 0;
    }
  }
}

// Thin windows (the 257th row or column next to tensor-core tiles): one warp
// per output, lanes split the reduction index, warp-sum of the signed counts.
template <int LW>
__global__ void __launch_bounds__(256) gemm_popc_thin_kernel(GemmProblem P) {
  const int lane = threadIdx.x & 31;
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t wm = P.m_hi - P.m_lo, wn = P.n_hi - P.n_lo;
  const int64_t total = P.batch * wm * wn;
  const int T = 1 << P.prec;
  const int WT = T >= 32 ? T / 32 : 1;
  for (int64_t o = wid; o < total; o += nwarps) {
    const int64_t slice = o / (wm * wn);
    const int64_t r = o % (wm * wn);
    const int64_t gm = P.m_lo + r / wn, gn = P.n_lo + r % wn;
    const int64_t slice_b = P.batch_b == 1 ? 0 : slice;
    const int64_t grow = slice * P.M + gm, brow = slice_b * P.N + gn;
    const int L = row_stream_len(P, slice, grow);
    if (L < 0) continue;  // warp-uniform
    int acc = 0;
    if (L > 0) {
      const int16_t *ca = P.qa.code + grow * P.ldk;
      const int16_t *cb = P.qb.code + brow * P.ldk;
      const int pd = P.pool_dims;
      int dm = lane % pd;  // pool row d mod pool_dims, advanced without a division
      for (int d = lane; d < (int)P.K; d += 32) {
        const int a = ca[d], b = cb[d];
        const int k = ((a < 0 ? -a : a) * L) >> P.prec;
        const uint32_t *st = P.stream_table + ((int64_t)dm * (T + 1) + (b < 0 ? -b : b)) * WT;
        dm += 32;
        while (dm >= pd) dm -= pd;
        int cnt = 0;
#pragma unroll
        for (int w = 0; w < LW; ++w) {
          const int lo = 32 * w;
          const uint32_t win = k >= lo + 32 ? 0xffffffffu : (k > lo ? ((1u << (k - lo)) - 1u) : 0u);
          cnt += __popc(win & st[w]);
        }
        acc += ((a < 0) != (b < 0) ? -cnt : cnt);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    }
    if (lane == 0) {
      float y = 0.0f;
      if (L > 0)
        y = sc_rescale(P.mode, P.prec, L, acc, P.K, P.qa.scale[grow], P.qa.zero[grow],
                       P.qa.rowsum[grow], P.qb.scale[brow], P.qb.zero[brow], P.qb.rowsum[brow]);
      if (P.bias) y = __fadd_rn(y, P.bias[gn]);
      store_out(P, grow * P.N + gn, y);
      if (P.acc_out) P.acc_out[grow * P.N + gn] = L > 0 ? acc : 0;
    }
  }
}

// Thin windows with a short reduction (K <= 512, e.g. the 257th row / column
// of Q@K^T and Attn@V): G lanes per output (G = 8 for K <= 128, else 32)
// split the reduction indices in chunks of 8 (lane j of a group takes
// indices 8 c .. 8 c + 7 for c = j, j + G, ..., one 16-byte load of each
// code row per chunk; the code rows are ldk = ceil8(K) long, padded with
// code 0, which counts nothing); the group's signed counts are summed with
// shuffles and its first lane rescales and stores.  Consecutive groups take
// consecutive columns of a row.  The count of index d is one 8-byte entry
// of the strip table, SW[d'][v][k / 32] = {stream word, prefix count}:
//   #{t < k : R[d'][t] < v} = count + popc(word & (2^(k % 32) - 1))
// (at k = 2^p the word is 0 and the mask empty).  Index math is 32-bit: the
// host launches this kernel when batch x strip < 2^31.
template <int G>
__global__ void __launch_bounds__(256) gemm_popc_thin_lane_kernel(GemmProblem P) {
  static_assert(G == 8 || G == 32, "lane groups of 8 or 32");
  const uint32_t wm = (uint32_t)(P.m_hi - P.m_lo), wn = (uint32_t)(P.n_hi - P.n_lo);
  const uint32_t wmn = wm * wn;
  const uint32_t total = (uint32_t)P.batch * wmn;
  const int T = 1 << P.prec;
  const int WT = T >= 32 ? T / 32 : 1;
  const int pd = P.pool_dims;
  const int nchunk = (int)(P.ldk >> 3);
  const int lane = threadIdx.x & 31;
  const int j = lane & (G - 1);
  constexpr uint32_t kGroupsPerWarp = 32 / G;
  const uint32_t gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const uint32_t nw = (gridDim.x * blockDim.x) >> 5;
  // the loop runs over warp-uniform bases, so every lane of a warp reaches
  // the shuffles below; groups past the end compute a copy of the last output
  // and store nothing
  for (uint32_t ow = gw * kGroupsPerWarp; ow < total; ow += nw * kGroupsPerWarp) {
    const uint32_t o = ow + (uint32_t)lane / G;
    const bool valid = o < total;
    const uint32_t oc = valid ? o : total - 1;
    const uint32_t sl = oc / wmn;
    const uint32_t r = oc - sl * wmn;
    const uint32_t rm = r / wn;
    const int64_t slice = sl;
    const int64_t gm = P.m_lo + rm, gn = P.n_lo + (r - rm * wn);
    const int64_t slice_b = P.batch_b == 1 ? 0 : slice;
    const int64_t grow = slice * P.M + gm, brow = slice_b * P.N + gn;
    const int L = row_stream_len(P, slice, grow);
    int acc = 0;
    if (L > 0) {
      const uint4 *ca = reinterpret_cast<const uint4 *>(P.qa.code + grow * P.ldk);
      const uint4 *cb = reinterpret_cast<const uint4 *>(P.qb.code + brow * P.ldk);
      for (int c = j; c < nchunk; c += G) {
        const uint4 av = __ldg(ca + c), bv = __ldg(cb + c);
        const uint32_t aw[4] = {av.x, av.y, av.z, av.w}, bw[4] = {bv.x, bv.y, bv.z, bv.w};
        int dm = (8 * c) % pd;  // pool row of the chunk's first index
        int a[8], b[8], k[8];
        uint2 e[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          a[i] = (i & 1) ? ((int)aw[i >> 1] >> 16) : (int)(int16_t)(aw[i >> 1] & 0xFFFFu);
          b[i] = (i & 1) ? ((int)bw[i >> 1] >> 16) : (int)(int16_t)(bw[i >> 1] & 0xFFFFu);
          // (k <= 2^p for every valid stream length; the clamp keeps the
          // table reads inside their rows whatever the per-row lengths hold)
          k[i] = min(((a[i] < 0 ? -a[i] : a[i]) * L) >> P.prec, T);
          const int v = b[i] < 0 ? -b[i] : b[i];
          e[i] = __ldg(P.strip_table + (dm * (T + 1) + v) * (WT + 1) + (k[i] >> 5));
          if (++dm == pd) dm = 0;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int cnt = (int)e[i].y +
                          __popc(__funnelshift_lc(0xffffffffu, 0u, (uint32_t)(k[i] & 31)) & e[i].x);
          acc += ((a[i] < 0) != (b[i] < 0) ? -cnt : cnt);
        }
      }
    }
#pragma unroll
    for (int off = G / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (!valid || j != 0 || L < 0) continue;
    float y = 0.0f;
    if (L > 0)
      y = sc_rescale(P.mode, P.prec, L, acc, P.K, P.qa.scale[grow], P.qa.zero[grow],
                     P.qa.rowsum[grow], P.qb.scale[brow], P.qb.zero[brow], P.qb.rowsum[brow]);
    if (P.bias) y = __fadd_rn(y, P.bias[gn]);
    store_out(P, grow * P.N + gn, y);
    if (P.acc_out) P.acc_out[grow * P.N + gn] = L > 0 ? acc : 0;
  }
}

cudaError_t launch_thin_lane(const GemmProblem &P, cudaStream_t s) {
  const int64_t total = P.batch * (P.m_hi - P.m_lo) * (P.n_hi - P.n_lo);
  const int G = P.K <= 128 ? 8 : 32;
  int64_t blocks = (total * G + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (G == 8)
    gemm_popc_thin_lane_kernel<8><<<(unsigned)blocks, 256, 0, s>>>(P);
  else
    gemm_popc_thin_lane_kernel<32><<<(unsigned)blocks, 256, 0, s>>>(P);
  return cudaGetLastError();
}

template <int LW>
cudaError_t launch_thin(const GemmProblem &P, cudaStream_t s) {
  const int64_t total = P.batch * (P.m_hi - P.m_lo) * (P.n_hi - P.n_lo);
  // (16-byte code loads: unsegmented code rows of ldk = ceil8(K) codes from
  // 16-byte aligned planes)
  const bool vec = P.nseg == 1 && (P.ldk & 7) == 0 &&
                   ((reinterpret_cast<uintptr_t>(P.qa.code) |
                     reinterpret_cast<uintptr_t>(P.qb.code)) & 15) == 0;
  if (P.K <= 512 && P.strip_table && vec && total < ((int64_t)1 << 31))
    return launch_thin_lane(P, s);
  int64_t blocks = (total + 7) / 8;  // 8 warps per block, one output per warp
  if (blocks > 148 * 32) blocks = 148 * 32;
  gemm_popc_thin_kernel<LW><<<(unsigned)blocks, 256, 0, s>>>(P);
  return cudaGetLastError();
}

template <int LW>
cudaError_t launch_lw(const GemmProblem &P, cudaStream_t s) {
  const size_t smem = PopcCfg<LW>::smem_bytes;
  cudaError_t e = cudaFuncSetAttribute(gemm_popc_kernel<LW>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)((P.n_hi - P.n_lo + BN - 1) / BN), (unsigned)((P.m_hi - P.m_lo + BM - 1) / BM),
            (unsigned)P.batch);
  gemm_popc_kernel<LW><<<grid, kThreads, smem, s>>>(P);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemm_popc(const GemmProblem &P, cudaStream_t s) {
  if (P.m_hi <= P.m_lo || P.n_hi <= P.n_lo || P.batch == 0) return cudaSuccess;
  // Words per stream: enough for the longest stream any row may use.
  const int T = 1 << P.prec;
  const int Lmax = (P.row_L || P.slice_L) ? T : P.stoc_len;
  const int lw = (Lmax + 31) / 32;
  const bool thin = P.nseg == 1 && (P.m_hi - P.m_lo <= 16 || P.n_hi - P.n_lo <= 16);
  if (thin) {
    if (lw <= 1) return launch_thin<1>(P, s);
    if (lw <= 2) return launch_thin<2>(P, s);
    if (lw <= 4) return launch_thin<4>(P, s);
    return launch_thin<8>(P, s);
  }
  if (lw <= 1) return launch_lw<1>(P, s);
  if (lw <= 2) return launch_lw<2>(P, s);
  if (lw <= 4) return launch_lw<4>(P, s);
  return launch_lw<8>(P, s);
}

}  // namespace scmp
