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

}  // namespace

cudaError_t launch_split_qkv(const void *qkv, int64_t B, int64_t N, int64_t H, int64_t D,
                             int elem_bytes, void *q, void *k, void *vt, cudaStream_t s) {
  if (B == 0 || N == 0 || H == 0 || D == 0) return cudaSuccess;
  if (elem_bytes == 2) return launch_split<uint16_t>(qkv, B, N, H, D, q, k, vt, s);
  return launch_split<uint32_t>(qkv, B, N, H, D, q, k, vt, s);
}

}  // namespace scmp
