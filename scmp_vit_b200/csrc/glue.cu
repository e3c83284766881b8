// Data movement around the attention SC matmuls: the fused qkv projection
// output [B, N, 3, H, D] is split into q, k [B, H, N, D] and v^T [B, H, D, N]
// in one pass, the layouts the per-head Q@K^T and per-row Attn@V calls read
// as plain contiguous slices.  Pure copies (2- or 4-byte elements), so the
// values are those of torch's permute / transpose.
#include <stdint.h>

#include "sc_common.cuh"

namespace scmp {
namespace {

// q and k: each (b, t, h) row of D elements moves as whole 16-byte units.
__global__ void split_qk_kernel(const uint4 *__restrict__ qkv, int64_t B, int64_t N, int64_t H,
                                int64_t units /* 16-byte units per row of D */,
                                uint4 *__restrict__ q, uint4 *__restrict__ k) {
  const int64_t per = B * N * H * units;  // units of one of q / k
  for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < 2 * per;
       u += (int64_t)gridDim.x * blockDim.x) {
    const int s = u >= per ? 1 : 0;
    int64_t r = u - s * per;
    const int64_t c = r % units;
    r /= units;
    const int64_t h = r % H;
    r /= H;
    const int64_t t = r % N;
    const int64_t b = r / N;
    const uint4 v = __ldg(qkv + (((b * N + t) * 3 + s) * H + h) * units + c);
    (s ? k : q)[((b * H + h) * N + t) * units + c] = v;
  }
}

// Any element size or alignment: one element per thread.
template <typename E>
__global__ void split_qk_elem_kernel(const E *__restrict__ qkv, int64_t B, int64_t N, int64_t H,
                                     int64_t D, E *__restrict__ q, E *__restrict__ k) {
  const int64_t per = B * N * H * D;
  for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < 2 * per;
       u += (int64_t)gridDim.x * blockDim.x) {
    const int s = u >= per ? 1 : 0;
    int64_t r = u - s * per;
    const int64_t d = r % D;
    r /= D;
    const int64_t h = r % H;
    r /= H;
    const int64_t t = r % N;
    const int64_t b = r / N;
    (s ? k : q)[((b * H + h) * N + t) * D + d] = qkv[(((b * N + t) * 3 + s) * H + h) * D + d];
  }
}

// v^T: block (b h, 64-token tile) stages v[b, t0 .. t0 + 63, 2, h, :] in
// shared memory (one column of padding against bank conflicts) and writes
// v^T rows d, 64 consecutive tokens at a time.  Warp w loads tokens w, w + 8,
// ... (its lanes along D) and stores rows d = w, w + 8, ... (its lanes along
// the tokens), so every access is coalesced and the index math stays 32-bit
// inside the tile.
constexpr int kVtTile = 64;

template <typename E>
__global__ void __launch_bounds__(256) split_vt_kernel(const E *__restrict__ qkv, int64_t N,
                                                       int64_t H, int D, E *__restrict__ vt) {
  extern __shared__ unsigned char smem_raw[];
  E *tile = reinterpret_cast<E *>(smem_raw);  // [kVtTile][D + 1]
  const int64_t bh = blockIdx.y;
  const int64_t b = bh / H, h = bh % H;
  const int64_t t0 = (int64_t)blockIdx.x * kVtTile;
  const int nt = (int)(N - t0 < kVtTile ? N - t0 : kVtTile);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ld = D + 1;
  for (int tt = warp; tt < nt; tt += 8) {
    const E *src = qkv + (((b * N + t0 + tt) * 3 + 2) * H + h) * (int64_t)D;
    for (int d = lane; d < D; d += 32) tile[tt * ld + d] = src[d];
  }
  __syncthreads();
  for (int d = warp; d < D; d += 8) {
    E *dst = vt + (bh * D + d) * N + t0;
    for (int tt = lane; tt < nt; tt += 32) dst[tt] = tile[tt * ld + d];
  }
}

template <typename E>
cudaError_t launch_split(const void *qkv, int64_t B, int64_t N, int64_t H, int64_t D, void *q,
                         void *k, void *vt, cudaStream_t s) {
  const int64_t row_bytes = D * (int64_t)sizeof(E);
  const bool vec = (row_bytes % 16) == 0 &&
                   ((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(q) |
                     reinterpret_cast<uintptr_t>(k)) & 15) == 0;
  const int64_t total = vec ? 2 * B * N * H * (row_bytes / 16) : 2 * B * N * H * D;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  if (vec)
    split_qk_kernel<<<(unsigned)blocks, 256, 0, s>>>(
        static_cast<const uint4 *>(qkv), B, N, H, row_bytes / 16, static_cast<uint4 *>(q),
        static_cast<uint4 *>(k));
  else
    split_qk_elem_kernel<E><<<(unsigned)blocks, 256, 0, s>>>(
        static_cast<const E *>(qkv), B, N, H, D, static_cast<E *>(q), static_cast<E *>(k));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const size_t smem = (size_t)kVtTile * (size_t)(D + 1) * sizeof(E);  // <= 66 KB (D <= 256)
  if (smem > 48 * 1024) {
    e = cudaFuncSetAttribute(split_vt_kernel<E>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem);
    if (e != cudaSuccess) return e;
  }
  const dim3 grid((unsigned)((N + kVtTile - 1) / kVtTile), (unsigned)(B * H));
  split_vt_kernel<E><<<grid, 256, smem, s>>>(static_cast<const E *>(qkv), N, H, (int)D,
                                               static_cast<E *>(vt));
  return cudaGetLastError();
}

// ---- the fp32 elementwise steps of a transformer block around its matmuls,
// fused.  Each operation is rounded on its own (no contraction), in the order
// of the unfused torch ops, so the results carry their bits.

// y = gelu(y + bias[c]) in place, gelu(t) = (t * 0.5) * (1 + erf(t * (1/sqrt 2)))
// (exact GELU), for an fc1 output without its bias.
__device__ __forceinline__ float gelu_exact(float t) {
  const float kInvSqrt2 = 0.70710678118654752440f;
  return __fmul_rn(__fmul_rn(t, 0.5f), __fadd_rn(1.0f, erff(__fmul_rn(t, kInvSqrt2))));
}
__global__ void bias_gelu_kernel(float *__restrict__ y, const float *__restrict__ bias,
                                 int64_t rows, int64_t cols) {
  const int64_t total = rows * cols;
  if ((cols & 3) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(bias) & 15) == 0) {
    float4 *y4 = reinterpret_cast<float4 *>(y);
    const float4 *b4 = reinterpret_cast<const float4 *>(bias);
    const int64_t c4 = cols >> 2;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (total >> 2);
         i += (int64_t)gridDim.x * blockDim.x) {
      float4 v = y4[i];
      const float4 b = __ldg(b4 + i % c4);
      v.x = gelu_exact(__fadd_rn(v.x, b.x));
      v.y = gelu_exact(__fadd_rn(v.y, b.y));
      v.z = gelu_exact(__fadd_rn(v.z, b.z));
      v.w = gelu_exact(__fadd_rn(v.w, b.w));
      y4[i] = v;
    }
    return;
  }
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] = gelu_exact(__fadd_rn(y[i], __ldg(bias + i % cols)));
}

// out = (x + (y [+ bias[c]]) * gamma[c]) [+ extra]: a branch output y (a
// matmul without its bias, or with it when bias is NULL) scaled by the layer
// scale and added to the residual x, then the optional extra term (a
// compensation output).  out may alias x or y.
__device__ __forceinline__ float scale_residual_one(float x, float y, float b, float g, float e,
                                                    bool has_b, bool has_e) {
  float t = has_b ? __fadd_rn(y, b) : y;
  t = __fadd_rn(x, __fmul_rn(t, g));
  return has_e ? __fadd_rn(t, e) : t;
}
__global__ void scale_residual_kernel(float *out, const float *x, const float *y,
                                      const float *__restrict__ bias,
                                      const float *__restrict__ gamma, const float *extra,
                                      int64_t rows, int64_t cols) {
  const int64_t total = rows * cols;
  const bool hb = bias != nullptr, he = extra != nullptr;
  const uintptr_t al = reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(x) |
                       reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(gamma) |
                       reinterpret_cast<uintptr_t>(bias) | reinterpret_cast<uintptr_t>(extra);
  if ((cols & 3) == 0 && (al & 15) == 0) {
    const int64_t c4 = cols >> 2;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (total >> 2);
         i += (int64_t)gridDim.x * blockDim.x) {
      const float4 xv = reinterpret_cast<const float4 *>(x)[i];
      const float4 yv = reinterpret_cast<const float4 *>(y)[i];
      const float4 g = __ldg(reinterpret_cast<const float4 *>(gamma) + i % c4);
      const float4 b = hb ? __ldg(reinterpret_cast<const float4 *>(bias) + i % c4)
                          : make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 e = he ? reinterpret_cast<const float4 *>(extra)[i]
                          : make_float4(0.f, 0.f, 0.f, 0.f);
      float4 o;
      o.x = scale_residual_one(xv.x, yv.x, b.x, g.x, e.x, hb, he);
      o.y = scale_residual_one(xv.y, yv.y, b.y, g.y, e.y, hb, he);
      o.z = scale_residual_one(xv.z, yv.z, b.z, g.z, e.z, hb, he);
      o.w = scale_residual_one(xv.w, yv.w, b.w, g.w, e.w, hb, he);
      reinterpret_cast<float4 *>(out)[i] = o;
    }
    return;
  }
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = i % cols;
    out[i] = scale_residual_one(x[i], y[i], hb ? bias[c] : 0.f, gamma[c], he ? extra[i] : 0.f,
                                hb, he);
  }
}

unsigned glue_blocks(int64_t n) {
  const int64_t b = (n + 255) / 256;
  return (unsigned)(b < 148 * 16 ? b : 148 * 16);
}

}  // namespace

cudaError_t launch_bias_gelu(float *y, const float *bias, int64_t rows, int64_t cols,
                             cudaStream_t s) {
  if (rows == 0 || cols == 0) return cudaSuccess;
  bias_gelu_kernel<<<glue_blocks(rows * cols / 4 + 1), 256, 0, s>>>(y, bias, rows, cols);
  return cudaGetLastError();
}

cudaError_t launch_scale_residual(float *out, const float *x, const float *y, const float *bias,
                                  const float *gamma, const float *extra, int64_t rows,
                                  int64_t cols, cudaStream_t s) {
  if (rows == 0 || cols == 0) return cudaSuccess;
  scale_residual_kernel<<<glue_blocks(rows * cols / 4 + 1), 256, 0, s>>>(out, x, y, bias, gamma,
                                                                           extra, rows, cols);
  return cudaGetLastError();
}

cudaError_t launch_split_qkv(const void *qkv, int64_t B, int64_t N, int64_t H, int64_t D,
                             int elem_bytes, void *q, void *k, void *vt, cudaStream_t s) {
  if (B == 0 || N == 0 || H == 0 || D == 0) return cudaSuccess;
  if (elem_bytes == 2) return launch_split<uint16_t>(qkv, B, N, H, D, q, k, vt, s);
  return launch_split<uint32_t>(qkv, B, N, H, D, q, k, vt, s);
}

}  // namespace scmp
