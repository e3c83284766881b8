// Throughput probes for the roofline denominators of the SC engines.
//
// Each probe runs a register-only loop of one instruction class on every SM
// and reports its sustained rate, measured with CUDA events:
//   kind 0: LOP3 (AND) + POPC on 32-bit words       -> bit-products per second
//   kind 1: mma.sync m16n8k256 b1 AND.POPC           -> bit-products per second
//   kind 2: mma.sync m16n8k32 s8 x s8 -> s32          -> multiply-adds per second
//   kind 3: tcgen05.mma kind::mxf4 M128 x N256 x K64   -> multiply-adds per second
//   kind 4: tcgen05.mma kind::mxf4 M128 x N64 x K64    -> multiply-adds per second
// A bit-product is one (m, n, d, t) term of the SC inner product, i.e. one
// AND + one counted bit; on the e2m1 tensor-core engine it is one
// multiply-add of operands in {-1, 0, +1}, so kinds 3 and 4 are the
// tensor-core engine's bit-product ceilings (the wide tiles' and Attn@V's).
#include <cuda_runtime.h>
#include <stdint.h>

#include "sc_common.cuh"

namespace {

constexpr int kIters = 4096;

__global__ void probe_popc(uint32_t seed, int iters, uint32_t *out) {
  uint32_t a0 = seed ^ threadIdx.x, a1 = a0 * 3u, a2 = a0 * 5u, a3 = a0 * 7u;
  uint32_t b0 = seed + blockIdx.x, b1 = b0 * 11u, b2 = b0 * 13u, b3 = b0 * 17u;
  int c0 = 0, c1 = 0, c2 = 0, c3 = 0, c4 = 0, c5 = 0, c6 = 0, c7 = 0;
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      c0 += __popc(a0 & b0); c1 += __popc(a1 & b1); c2 += __popc(a2 & b2); c3 += __popc(a3 & b3);
      c4 += __popc(a0 & b1); c5 += __popc(a1 & b2); c6 += __popc(a2 & b3); c7 += __popc(a3 & b0);
      a0 += 0x9E3779B9u; b3 ^= a0;  // keep the operands live and changing
    }
  }
  out[blockIdx.x * blockDim.x + threadIdx.x] = c0 + c1 + c2 + c3 + c4 + c5 + c6 + c7;
}

__global__ void probe_mma_b1(uint32_t seed, int iters, uint32_t *out) {
  uint32_t A0 = seed ^ threadIdx.x, A1 = A0 * 3u, A2 = A0 * 5u, A3 = A0 * 7u;
  uint32_t B0 = seed + blockIdx.x, B1 = B0 * 11u;
  int d[4][4] = {};
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      asm volatile(
          "mma.sync.aligned.m16n8k256.row.col.s32.b1.b1.s32.and.popc "
          "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
          : "+r"(d[u][0]), "+r"(d[u][1]), "+r"(d[u][2]), "+r"(d[u][3])
          : "r"(A0), "r"(A1), "r"(A2), "r"(A3), "r"(B0), "r"(B1));
    }
  }
  int s = 0;
#pragma unroll
  for (int u = 0; u < 4; ++u) s += d[u][0] + d[u][1] + d[u][2] + d[u][3];
  out[blockIdx.x * blockDim.x + threadIdx.x] = (uint32_t)s;
}

__global__ void probe_mma_s8(uint32_t seed, int iters, uint32_t *out) {
  uint32_t A0 = seed ^ threadIdx.x, A1 = A0 * 3u, A2 = A0 * 5u, A3 = A0 * 7u;
  uint32_t B0 = seed + blockIdx.x, B1 = B0 * 11u;
  int d[4][4] = {};
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      asm volatile(
          "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
          "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
          : "+r"(d[u][0]), "+r"(d[u][1]), "+r"(d[u][2]), "+r"(d[u][3])
          : "r"(A0), "r"(A1), "r"(A2), "r"(A3), "r"(B0), "r"(B1));
    }
  }
  int s = 0;
#pragma unroll
  for (int u = 0; u < 4; ++u) s += d[u][0] + d[u][1] + d[u][2] + d[u][3];
  out[blockIdx.x * blockDim.x + threadIdx.x] = (uint32_t)s;
}

// kinds 3 / 4: the e2m1 MMA issued back to back on every SM (MACs per second)
int probe_mxf4(int n, int sms, double *ops_per_second) {
  constexpr int kMmaIters = 2048;
  unsigned int *err = nullptr;
  if (cudaMalloc(&err, sizeof(unsigned int)) != cudaSuccess) return SCMP_ECUDA;
  cudaMemset(err, 0, sizeof(unsigned int));
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaError_t e = scmp::launch_probe_mma_mxf4(n, 16, sms, err, 0);  // warm-up
  if (e == cudaSuccess) {
    cudaEventRecord(e0);
    e = scmp::launch_probe_mma_mxf4(n, kMmaIters, sms, err, 0);
    cudaEventRecord(e1);
  }
  if (e == cudaSuccess) e = cudaEventSynchronize(e1);
  float ms = 0.f;
  cudaEventElapsedTime(&ms, e0, e1);
  unsigned int flag = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&flag, err, sizeof(flag), cudaMemcpyDeviceToHost);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaFree(err);
  if (e != cudaSuccess || flag != 0 || ms <= 0.f) return e != cudaSuccess ? SCMP_ECUDA : SCMP_ETIMEOUT;
  *ops_per_second = 4.0 * kMmaIters * 128.0 * n * 64.0 * sms / (ms * 1e-3);
  return SCMP_OK;
}

}  // namespace

extern "C" SCMP_API int scmp_probe_int_peak(int kind, double *ops_per_second) {
  if (!ops_per_second || kind < 0 || kind > 4) return SCMP_EINVAL;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return SCMP_ECUDA;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return SCMP_ECUDA;
  if (kind >= 3) return probe_mxf4(kind == 3 ? 256 : 64, sms, ops_per_second);
  const int threads = 256, blocks = sms * 8;
  uint32_t *out = nullptr;
  if (cudaMalloc(&out, sizeof(uint32_t) * threads * blocks) != cudaSuccess) return SCMP_ECUDA;
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  auto launch = [&](int iters) {
    if (kind == 0) probe_popc<<<blocks, threads>>>(12345u, iters, out);
    else if (kind == 1) probe_mma_b1<<<blocks, threads>>>(12345u, iters, out);
    else probe_mma_s8<<<blocks, threads>>>(12345u, iters, out);
  };
  launch(64);  // warm-up
  cudaEventRecord(e0);
  launch(kIters);
  cudaEventRecord(e1);
  cudaError_t err = cudaEventSynchronize(e1);
  float ms = 0.f;
  cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaFree(out);
  if (err != cudaSuccess || cudaGetLastError() != cudaSuccess || ms <= 0.f) return SCMP_ECUDA;
  const double per_iter_thread = kind == 0 ? 32.0 * 32.0  // 32 popcounts x 32 bits
                                           : 4.0 * (kind == 1 ? 16.0 * 8 * 256 : 16.0 * 8 * 32) / 32.0;
  *ops_per_second = per_iter_thread * (double)kIters * threads * blocks / (ms * 1e-3);
  return SCMP_OK;
}
