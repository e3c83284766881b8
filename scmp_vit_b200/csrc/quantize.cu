// Quantisation of SC operands and the per-pool stream table.
//
// Bit-exact restatement of sco_quantize in oracle/sc_oracle.c: IEEE fp32
// divide/multiply (no contraction), round-half-even, 1e-6 floor on the range
// (reference sc_integration/sc_linear.py:95-111).
#include <type_traits>

#include "sc_common.cuh"

namespace scmp {
namespace {

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
template <typename T>
__device__ __forceinline__ float ldx(const T *p);
template <>
__device__ __forceinline__ float ldx<float>(const float *p) {
  return __ldg(p);
}
template <>
__device__ __forceinline__ float ldx<__nv_bfloat16>(const __nv_bfloat16 *p) {
  return __bfloat162float(__ldg(p));
}

__device__ __forceinline__ int warp_sum(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
// Reductions over the LPR lanes that share a row (aligned groups of a warp).
template <int LPR>
__device__ __forceinline__ float group_max(float v) {
#pragma unroll
  for (int o = LPR / 2; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
template <int LPR>
__device__ __forceinline__ float group_min(float v) {
#pragma unroll
  for (int o = LPR / 2; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
template <int LPR>
__device__ __forceinline__ int group_sum(int v) {
#pragma unroll
  for (int o = LPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// LPR lanes per row (32, or 8 for short rows): (max|x|, -) for bipolar,
// (min x, max x) for unipolar.
template <typename T, int LPR>
__global__ void row_stats_kernel(const T *__restrict__ x, int64_t rows, int64_t K, int mode,
                                 float2 *__restrict__ stat) {
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / LPR;
  const int lane = threadIdx.x % LPR;
  const bool active = row < rows;  // inactive lanes still take part in the shuffles
  const T *xr = x + (active ? row : 0) * K;
  const int64_t kk = active ? K : 0;
  float lo = INFINITY, hi = -INFINITY;
  if constexpr (!std::is_same<T, float>::value || LPR != 32) {
    for (int64_t i = lane; i < kk; i += LPR) {
      const float v = ldx(xr + i);
      if (mode == SCMP_BIPOLAR) {
        hi = fmaxf(hi, fabsf(v));
      } else {
        lo = fminf(lo, v);
        hi = fmaxf(hi, v);
      }
    }
  } else if ((K & 3) == 0 && (((uintptr_t)xr) & 15) == 0) {
    const float4 *x4 = reinterpret_cast<const float4 *>(xr);
    for (int64_t i = lane; i < (kk >> 2); i += 32) {
      float4 v = __ldg(x4 + i);
      if (mode == SCMP_BIPOLAR) {
        hi = fmaxf(hi, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
      } else {
        lo = fminf(lo, fminf(fminf(v.x, v.y), fminf(v.z, v.w)));
        hi = fmaxf(hi, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
      }
    }
  } else {
    for (int64_t i = lane; i < kk; i += 32) {
      float v = __ldg(xr + i);
      if (mode == SCMP_BIPOLAR) {
        hi = fmaxf(hi, fabsf(v));
      } else {
        lo = fminf(lo, v);
        hi = fmaxf(hi, v);
      }
    }
  }
  hi = group_max<LPR>(hi);
  lo = group_min<LPR>(lo);
  if (active && lane == 0) stat[row] = make_float2(lo, hi);
}

// Scale, inverse scale and zero point of one group from its min / max.
__device__ __forceinline__ void group_scale_of(float lo, float hi, int mode, int prec,
                                               float &scale, float &inv, int32_t &zero) {
  if (mode == SCMP_BIPOLAR) {
    const float qmax = (float)((1 << (prec - 1)) - 1);
    const float amax = hi > 1e-6f ? hi : 1e-6f;
    scale = __fdiv_rn(amax, qmax);
    inv = __fdiv_rn(qmax, amax);
    zero = 0;
  } else {
    const float qmax = (float)((1 << prec) - 1);
    float rng = __fsub_rn(hi, lo);
    if (!(rng > 1e-6f)) rng = 1e-6f;
    inv = __fdiv_rn(qmax, rng);
    scale = __fdiv_rn(rng, qmax);
    zero = __float2int_rn(__fmul_rn(-lo, inv));
  }
}

// Scale of one group (shared by both group kernels).
__device__ __forceinline__ void write_group_scale(int64_t grp, float lo, float hi, int mode,
                                                  int prec, float *__restrict__ gscale,
                                                  float *__restrict__ ginv,
                                                  int32_t *__restrict__ gzero) {
  float scale, inv;
  int32_t zero;
  group_scale_of(lo, hi, mode, prec, scale, inv, zero);
  gscale[grp] = scale;
  ginv[grp] = inv;
  gzero[grp] = zero;
}

// Small groups (per-row scaling, a few rows per group): one thread per group.
__global__ void group_stats_small_kernel(const float2 *__restrict__ stat, GroupShape g, int mode,
                                         int prec, float *__restrict__ gscale,
                                         float *__restrict__ ginv, int32_t *__restrict__ gzero) {
  for (int64_t grp = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; grp < g.ngroups;
       grp += (int64_t)gridDim.x * blockDim.x) {
    const int64_t slice = grp / g.groups_per_slice;
    const int64_t j = grp % g.groups_per_slice;
    const int64_t r0 = slice * g.slice_rows + j * g.group_rows;
    int64_t r1 = r0 + g.group_rows;
    const int64_t slice_end = (slice + 1) * g.slice_rows;
    if (r1 > slice_end) r1 = slice_end;
    float lo = INFINITY, hi = -INFINITY;
    for (int64_t r = r0; r < r1; ++r) {
      const float2 s = stat[r];
      lo = fminf(lo, s.x);
      hi = fmaxf(hi, s.y);
    }
    write_group_scale(grp, lo, hi, mode, prec, gscale, ginv, gzero);
  }
}

// Large groups: one block per scale group.
__global__ void __launch_bounds__(1024) group_stats_kernel(const float2 *__restrict__ stat, GroupShape g, int mode,
                                   int prec, float *__restrict__ gscale,
                                   float *__restrict__ ginv, int32_t *__restrict__ gzero) {
  const int64_t grp = blockIdx.x;
  if (grp >= g.ngroups) return;
  const int64_t slice = grp / g.groups_per_slice;
  const int64_t j = grp % g.groups_per_slice;
  const int64_t r0 = slice * g.slice_rows + j * g.group_rows;
  int64_t r1 = r0 + g.group_rows;
  const int64_t slice_end = (slice + 1) * g.slice_rows;
  if (r1 > slice_end) r1 = slice_end;
  float lo = INFINITY, hi = -INFINITY;
#pragma unroll 4
  for (int64_t r = r0 + threadIdx.x; r < r1; r += blockDim.x) {
    float2 s = stat[r];
    lo = fminf(lo, s.x);
    hi = fmaxf(hi, s.y);
  }
  __shared__ float slo[32], shi[32];
  lo = warp_min(lo);
  hi = warp_max(hi);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { slo[w] = lo; shi[w] = hi; }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    lo = lane < nw ? slo[lane] : INFINITY;
    hi = lane < nw ? shi[lane] : -INFINITY;
    lo = warp_min(lo);
    hi = warp_max(hi);
    if (lane == 0) write_group_scale(grp, lo, hi, mode, prec, gscale, ginv, gzero);
  }
}

// LPR lanes per row: signed codes, per-row scale/zero, magnitude row sum.
// Codes are written with row stride ldc >= K; indices K .. ldc-1 get code 0,
// which contributes nothing to any count (zero window, zero threshold).
template <typename T, int LPR>
__global__ void quantize_kernel(const T *__restrict__ x, GroupShape g, int64_t K, int64_t ldc,
                                int mode, int prec, const float *__restrict__ gscale,
                                const float *__restrict__ ginv, const int32_t *__restrict__ gzero,
                                int16_t *__restrict__ code, float *__restrict__ rscale,
                                int32_t *__restrict__ rzero, int32_t *__restrict__ rsum) {
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / LPR;
  const int lane = threadIdx.x % LPR;
  const bool active = row < g.rows;  // inactive lanes still take part in the shuffles
  const int64_t r = active ? row : 0;
  const int64_t grp = group_of_row(g, r);
  const float inv = ginv[grp];
  const int32_t z = gzero[grp];
  const T *xr = x + r * K;
  int16_t *cr = code + r * ldc;
  const int64_t kk = active ? K : 0;
  if (active)
    for (int64_t i = K + lane; i < ldc; i += LPR) cr[i] = 0;
  int acc = 0;
  if (mode == SCMP_BIPOLAR) {
    const int iq = (1 << (prec - 1)) - 1;
    for (int64_t i = lane; i < kk; i += LPR) {
      int q = __float2int_rn(__fmul_rn(ldx(xr + i), inv));
      q = max(-iq, min(iq, q));
      cr[i] = (int16_t)(2 * q);
      acc += 2 * abs(q);
    }
  } else {
    const int iq = (1 << prec) - 1;
    for (int64_t i = lane; i < kk; i += LPR) {
      int q = __float2int_rn(__fmul_rn(ldx(xr + i), inv)) + z;
      q = max(0, min(iq, q));
      cr[i] = (int16_t)q;
      acc += q;
    }
  }
  acc = group_sum<LPR>(acc);
  if (active && lane == 0) {
    rscale[row] = gscale[grp];
    rzero[row] = z;
    rsum[row] = acc;
  }
}

// One-row scale groups (per-row scaling with group size 1), fused: the row's
// min / max, its scale and its codes in one launch.  The LPR lanes of a row
// read it twice, the second time from L1; the arithmetic and its order are
// those of row_stats_kernel + group_stats_small_kernel + quantize_kernel, so
// the codes and scales are identical.
template <typename T, int LPR>
__global__ void quantize_rows_kernel(const T *__restrict__ x, int64_t rows, int64_t K,
                                     int64_t ldc, int mode, int prec,
                                     int16_t *__restrict__ code, float *__restrict__ rscale,
                                     int32_t *__restrict__ rzero, int32_t *__restrict__ rsum) {
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / LPR;
  const int lane = threadIdx.x % LPR;
  const bool active = row < rows;  // inactive lanes still take part in the shuffles
  const int64_t r = active ? row : 0;
  const T *xr = x + r * K;
  int16_t *cr = code + r * ldc;
  const int64_t kk = active ? K : 0;
  // VEC elements per 16-byte load (4 fp32 or 8 bf16) when the row, its
  // length and the code row allow it; one element at a time otherwise
  constexpr int VEC = std::is_same<T, float>::value ? 4 : 8;
  const bool vec = (K % VEC) == 0 && (ldc % VEC) == 0 && ((uintptr_t)xr & 15) == 0 &&
                   ((uintptr_t)cr & (2 * VEC - 1)) == 0;
  auto load_vec = [&](int64_t i, float (&v)[VEC]) {
    const uint4 w = __ldg(reinterpret_cast<const uint4 *>(xr + i));
    if constexpr (std::is_same<T, float>::value) {
      v[0] = __uint_as_float(w.x);
      v[1] = __uint_as_float(w.y);
      v[2] = __uint_as_float(w.z);
      v[3] = __uint_as_float(w.w);
    } else {
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[2 * j] = __uint_as_float(ws[j] << 16);  // bf16 -> fp32, exact
        v[2 * j + 1] = __uint_as_float(ws[j] & 0xFFFF0000u);
      }
    }
  };
  float lo = INFINITY, hi = -INFINITY;
  if (vec) {
    for (int64_t i = lane * VEC; i < kk; i += LPR * VEC) {
      float v[VEC];
      load_vec(i, v);
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        if (mode == SCMP_BIPOLAR) {
          hi = fmaxf(hi, fabsf(v[j]));
        } else {
          lo = fminf(lo, v[j]);
          hi = fmaxf(hi, v[j]);
        }
      }
    }
  } else {
    for (int64_t i = lane; i < kk; i += LPR) {
      const float v = ldx(xr + i);
      if (mode == SCMP_BIPOLAR) {
        hi = fmaxf(hi, fabsf(v));
      } else {
        lo = fminf(lo, v);
        hi = fmaxf(hi, v);
      }
    }
  }
  hi = group_max<LPR>(hi);
  lo = group_min<LPR>(lo);
  float scale, inv;
  int32_t z;
  group_scale_of(lo, hi, mode, prec, scale, inv, z);
  if (active)
    for (int64_t i = K + lane; i < ldc; i += LPR) cr[i] = 0;
  int acc = 0;
  if (vec) {
    const bool bip = mode == SCMP_BIPOLAR;
    const int iq = bip ? (1 << (prec - 1)) - 1 : (1 << prec) - 1;
    for (int64_t i = lane * VEC; i < kk; i += LPR * VEC) {
      float v[VEC];
      load_vec(i, v);
      uint32_t p[VEC / 2];
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        int q = __float2int_rn(__fmul_rn(v[j], inv));
        int c;
        if (bip) {
          q = max(-iq, min(iq, q));
          c = 2 * q;
          acc += 2 * abs(q);
        } else {
          q = max(0, min(iq, q + z));
          c = q;
          acc += q;
        }
        if (j & 1)
          p[j >> 1] |= (uint32_t)(uint16_t)c << 16;
        else
          p[j >> 1] = (uint16_t)c;
      }
      if constexpr (VEC == 4)
        *reinterpret_cast<uint2 *>(cr + i) = make_uint2(p[0], p[1]);
      else
        *reinterpret_cast<uint4 *>(cr + i) = make_uint4(p[0], p[1], p[2], p[3]);
    }
  } else if (mode == SCMP_BIPOLAR) {
    const int iq = (1 << (prec - 1)) - 1;
    for (int64_t i = lane; i < kk; i += LPR) {
      int q = __float2int_rn(__fmul_rn(ldx(xr + i), inv));
      q = max(-iq, min(iq, q));
      cr[i] = (int16_t)(2 * q);
      acc += 2 * abs(q);
    }
  } else {
    const int iq = (1 << prec) - 1;
    for (int64_t i = lane; i < kk; i += LPR) {
      int q = __float2int_rn(__fmul_rn(ldx(xr + i), inv)) + z;
      q = max(0, min(iq, q));
      cr[i] = (int16_t)q;
      acc += q;
    }
  }
  acc = group_sum<LPR>(acc);
  if (active && lane == 0) {
    rscale[row] = scale;
    rzero[row] = z;
    rsum[row] = acc;
  }
}

// Per-slice scale groups of short rows (per-head scaling of attention
// slices: 257 rows of 64), fused: one block per slice holds the whole slice
// in registers (up to kSliceVec float4 per thread, 16-byte loads issued
// together), takes its max |x| (or min / max), the slice's scale, and writes
// the codes and row records from the registers.  Rows are K = 4 R elements
// with R dividing 32, so each row's float4s sit in R adjacent lanes, which
// sum its codes with shuffles.  Same arithmetic as row_stats_kernel +
// group_stats_kernel + quantize_kernel (min / max are exact in any order), so
// the codes and scales are identical.
constexpr int kSliceVec = 20;
template <int R>
__global__ void __launch_bounds__(256) quantize_slices_kernel(
    const float *__restrict__ x, int64_t rows_per_slice, int mode, int prec,
    int16_t *__restrict__ code, float *__restrict__ rscale, int32_t *__restrict__ rzero,
    int32_t *__restrict__ rsum) {
  constexpr int K = 4 * R;
  const int64_t slice = blockIdx.x;
  const int nvec = (int)(rows_per_slice * R);  // float4s in the slice
  const float4 *xs = reinterpret_cast<const float4 *>(x + slice * rows_per_slice * K);
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const bool bip = mode == SCMP_BIPOLAR;
  float4 v[kSliceVec];
#pragma unroll
  for (int i = 0; i < kSliceVec; ++i) {
    const int f = t + 256 * i;
    v[i] = f < nvec ? __ldg(xs + f) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float lo = INFINITY, hi = -INFINITY;
#pragma unroll
  for (int i = 0; i < kSliceVec; ++i) {
    if (t + 256 * i < nvec) {
      const float e[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (bip) {
          hi = fmaxf(hi, fabsf(e[j]));
        } else {
          lo = fminf(lo, e[j]);
          hi = fmaxf(hi, e[j]);
        }
      }
    }
  }
  __shared__ float slo[8], shi[8];
  lo = warp_min(lo);
  hi = warp_max(hi);
  if (lane == 0) {
    slo[warp] = lo;
    shi[warp] = hi;
  }
  __syncthreads();
  lo = INFINITY;
  hi = -INFINITY;
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    lo = fminf(lo, slo[w]);
    hi = fmaxf(hi, shi[w]);
  }
  float sc, inv;
  int32_t z;
  group_scale_of(lo, hi, mode, prec, sc, inv, z);
  const int iq = bip ? (1 << (prec - 1)) - 1 : (1 << prec) - 1;
  uint2 *cs = reinterpret_cast<uint2 *>(code + slice * rows_per_slice * K);
  const int64_t row0 = slice * rows_per_slice;
#pragma unroll
  for (int i = 0; i < kSliceVec; ++i) {
    const int f = t + 256 * i;
    if (256 * i >= nvec) break;  // block-uniform
    const bool ok = f < nvec;
    const float e[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
    int c[4], acc = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int q = __float2int_rn(__fmul_rn(e[j], inv));
      if (bip) {
        q = max(-iq, min(iq, q));
        c[j] = 2 * q;
        acc += 2 * abs(q);
      } else {
        q = max(0, min(iq, q + z));
        c[j] = q;
        acc += q;
      }
    }
    if (ok)
      cs[f] = make_uint2(((uint32_t)(uint16_t)c[0]) | ((uint32_t)(uint16_t)c[1] << 16),
                         ((uint32_t)(uint16_t)c[2]) | ((uint32_t)(uint16_t)c[3] << 16));
    // a row's R float4s are lanes f - f % R .. + R - 1 of this warp
#pragma unroll
    for (int o = R / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (ok && f % R == 0) {
      const int64_t r = row0 + f / R;
      rscale[r] = sc;
      rzero[r] = z;
      rsum[r] = acc;
    }
  }
}

// Softmax of scale * x along rows of K (32 < K <= 1024) values, then the
// per-row quantisation of the probabilities (the a operand of a per-row
// Attn@V call), in one pass with one warp per row.  The softmax repeats the
// arithmetic of torch.softmax's warp-per-row kernel for fp32 rows of up to
// 1024 values, so the probabilities carry the same bits: lane l holds the
// elements l + 32 i (i < NI; -inf past K; torch holds NI = the next power
// of two >= K, over 32, and any NI >= K / 32 gives the same sums); the row maximum is taken by lane, in i order, then by xor
// butterfly; e = expf(v - max) is summed by lane in i order starting from
// 0, then by xor butterfly; p = e / sum (IEEE division).  The quantisation
// is that of quantize_rows_kernel (group_scale_of, round half to even, the
// same clamps and row sums), so codes and row records are identical to
// quantising the probabilities after torch.softmax.  probs (nullable)
// receives the probabilities.
template <int NI>
__global__ void __launch_bounds__(256) softmax_quantize_kernel(
    const float *__restrict__ x, int64_t rows, int K, float scale, int mode, int prec,
    int64_t ldc, int16_t *__restrict__ code, float *__restrict__ rscale,
    int32_t *__restrict__ rzero, int32_t *__restrict__ rsum, float *__restrict__ probs) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const bool bip = mode == SCMP_BIPOLAR;
  const int iq = bip ? (1 << (prec - 1)) - 1 : (1 << prec) - 1;
  for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += nwarps) {
    const float *xr = x + r * K;
    float v[NI];
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const int idx = lane + 32 * i;
      v[i] = idx < K ? __fmul_rn(__ldg(xr + idx), scale) : -INFINITY;
    }
    float mx = v[0];
#pragma unroll
    for (int i = 0; i < NI; ++i) mx = mx > v[i] ? mx : v[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float t = __shfl_xor_sync(0xffffffffu, mx, o);
      mx = mx < t ? t : mx;
    }
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      v[i] = expf(__fsub_rn(v[i], mx));
      sum = __fadd_rn(sum, v[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
    float lo = INFINITY, hi = -INFINITY;
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const int idx = lane + 32 * i;
      if (idx < K) {
        v[i] = __fdiv_rn(v[i], sum);
        if (probs) probs[r * K + idx] = v[i];
        if (bip) {
          hi = fmaxf(hi, fabsf(v[i]));
        } else {
          lo = fminf(lo, v[i]);
          hi = fmaxf(hi, v[i]);
        }
      }
    }
    hi = warp_max(hi);
    lo = warp_min(lo);
    float sc, inv;
    int32_t z;
    group_scale_of(lo, hi, mode, prec, sc, inv, z);
    int16_t *cr = code + r * ldc;
    int acc = 0;
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const int idx = lane + 32 * i;
      if (idx < K) {
        int q = __float2int_rn(__fmul_rn(v[i], inv));
        if (bip) {
          q = max(-iq, min(iq, q));
          cr[idx] = (int16_t)(2 * q);
          acc += 2 * abs(q);
        } else {
          q = max(0, min(iq, q + z));
          cr[idx] = (int16_t)q;
          acc += q;
        }
      }
    }
    for (int64_t i = K + lane; i < ldc; i += 32) cr[i] = 0;
    acc = warp_sum(acc);
    if (lane == 0) {
      rscale[r] = sc;
      rzero[r] = z;
      rsum[r] = acc;
    }
  }
}

// ST[d][v][w]: bit j of word w = [R[d][32w+j] < v] for 32w+j < 2^p; with
// strips != NULL also the thin strips' table SW[d][v][w] = {ST[d][v][w],
// #{t < 32 w : R[d][t] < v}} for w = 0 .. WT (word 0 at w = WT), one 8-byte
// entry per lookup.  One thread per word; the WT words of a (d, v) sit in
// adjacent lanes, which scan their popcounts with shuffles (WT divides 32,
// so a group never spans two warps, and the loop runs over warp-aligned bases
// so that every lane reaches the shuffles).
__global__ void stream_table_kernel(const uint8_t *__restrict__ pool, int pool_dims, int prec,
                                    uint32_t *__restrict__ table, uint2 *__restrict__ strips) {
  const int T = 1 << prec;
  const int WT = T >= 32 ? T / 32 : 1;
  const int64_t total = (int64_t)pool_dims * (T + 1) * WT;
  const int lane = threadIdx.x & 31;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t base = (((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5) << 5; base < total;
       base += warps << 5) {
    const int64_t i = base + lane;
    const bool valid = i < total;
    const int w = (int)(i % WT);
    const int64_t dv = i / WT;
    const int v = (int)(dv % (T + 1));
    const int64_t d = dv / (T + 1);
    uint32_t word = 0;
    if (valid) {
      const uint8_t *R = pool + d * T + 32 * w;
#pragma unroll 8
      for (int j = 0; j < 32; ++j)
        if (32 * w + j < T && (int)R[j] < v) word |= 1u << j;
      table[i] = word;
    }
    if (strips) {
      const int c = __popc(word);
      int incl = c;
      for (int off = 1; off < WT; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, off, WT);
        if (w >= off) incl += y;
      }
      if (valid) {
        strips[dv * (WT + 1) + w] = make_uint2(word, (uint32_t)(incl - c));
        if (w == WT - 1) strips[dv * (WT + 1) + WT] = make_uint2(0u, (uint32_t)incl);
      }
    }
  }
}

// PC[d][t] = 0x7F - (R[d][t] >> shift).  The tensor-core engine forms the
// stream byte 0x7F + u - (R >> shift) for a threshold u < 128: its top bit is
// [R >> shift < u], with no borrow into the neighbouring byte.
// Written with row stride Lp = 2^lp_log2 <= 2^prec (the padded stream
// length; positions t >= Lp are never read).  Rows past the pool (reduction
// indices of zero padding) hold 0x7F: with a zero threshold they produce no
// stream bits.
__global__ void pool_complement_kernel(const uint8_t *__restrict__ pool, int pool_dims,
                                       int64_t rows, int prec, int lp_log2, int shift,
                                       int nibble_pairs, uint8_t *__restrict__ out) {
  const int64_t bytes = rows << lp_log2;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < bytes;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t d = i >> lp_log2;
    const int64_t slot = i & ((1 << lp_log2) - 1);
    // group slot j < 4 holds position 2 j, slot j >= 4 position 2 (j - 4) + 1
    const int64_t t = nibble_pairs ? (slot & ~7) + (((slot & 3) << 1) | ((slot >> 2) & 1)) : slot;
    out[i] = d < pool_dims ? (uint8_t)(0x7F - (pool[(d << prec) + t] >> shift)) : (uint8_t)0x7F;
  }
}

__device__ __forceinline__ uint32_t prmt_sign(uint32_t a) {
  uint32_t r;
  asm("prmt.b32 %0, %1, 0, 0xBA98;" : "=r"(r) : "r"(a));
  return r;
}

// Prepacked b operand bytes at Lp = 2^prec, one thread per 16-byte chunk:
// byte t of reduction index d of row n is sigma * [R[d][t] >> shift < u]
// with u = |c| >> shift, formed exactly as the tensor-core row producers
// form it (u * 0x01010101 + PC, sign-replicating byte permute, AND with
// 0x01010101 or 0xFFFFFFFF).  pool_comp rows are 2^prec bytes apart.
__global__ void pack_b_streams_kernel(const int16_t *__restrict__ code, int64_t N, int64_t ldk,
                                      int prec, int shift, int64_t pool_period,
                                      const uint8_t *__restrict__ pool_comp,
                                      uint8_t *__restrict__ out) {
  const int64_t row_bytes = ldk << prec;
  const int64_t per_row = row_bytes >> 4;
  const int64_t total = N * per_row;
  const int64_t tmask = (1 << prec) - 1;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / per_row;
    const int64_t pos = (i % per_row) << 4;
    const int64_t d = pos >> prec;
    const int c = code[n * ldk + d];
    const uint32_t u = (uint32_t)(abs(c) >> shift);
    const uint32_t sm = (uint32_t)(c >> 31) | 0x01010101u;
    const int64_t prow = pool_period > 0 ? d % pool_period : d;
    const uint4 pc =
        *reinterpret_cast<const uint4 *>(pool_comp + (prow << prec) + (pos & tmask));
    uint4 w;
    w.x = prmt_sign(u * 0x01010101u + pc.x) & sm;
    w.y = prmt_sign(u * 0x01010101u + pc.y) & sm;
    w.z = prmt_sign(u * 0x01010101u + pc.z) & sm;
    w.w = prmt_sign(u * 0x01010101u + pc.w) & sm;
    *reinterpret_cast<uint4 *>(out + n * row_bytes + pos) = w;
  }
}

// e2m1 form: one thread per 16 output bytes = 32 positions of one reduction
// index.  Nibble i of word w is position 8 w + i; each nibble is
// sigma * [R >> shift < u] as 0x2 (+1), 0xA (-1) or 0x0, formed as the e2m1
// pair producers form it from even / odd position complements.
__global__ void pack_b_streams_e2m1_kernel(const int16_t *__restrict__ code, int64_t N,
                                           int64_t ldk, int prec, int shift, int64_t pool_period,
                                           const uint8_t *__restrict__ pool_comp,
                                           uint8_t *__restrict__ out) {
  const int64_t row_bytes = (ldk << prec) >> 1;
  const int64_t per_row = row_bytes >> 4;
  const int64_t total = N * per_row;
  const int64_t tmask = (1 << prec) - 1;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / per_row;
    const int64_t pos = (i % per_row) << 5;  // first of 32 positions
    const int64_t d = pos >> prec;
    const int c = code[n * ldk + d];
    const uint32_t u = (uint32_t)(abs(c) >> shift);
    const uint32_t pat = c < 0 ? 0xAAAAAAAAu : 0x22222222u;
    const int64_t prow = pool_period > 0 ? d % pool_period : d;
    const uint4 *pc = reinterpret_cast<const uint4 *>(pool_comp + (prow << prec) + (pos & tmask));
    const uint4 p0 = pc[0], p1 = pc[1];
    const uint32_t w8[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
    uint32_t r[4];
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      uint32_t ev, od;  // complements of positions 8g + {0, 2, 4, 6} / {1, 3, 5, 7}
      asm("prmt.b32 %0, %1, %2, 0x6420;" : "=r"(ev) : "r"(w8[2 * g]), "r"(w8[2 * g + 1]));
      asm("prmt.b32 %0, %1, %2, 0x7531;" : "=r"(od) : "r"(w8[2 * g]), "r"(w8[2 * g + 1]));
      const uint32_t e = prmt_sign(u * 0x01010101u + ev);
      const uint32_t o = prmt_sign(u * 0x01010101u + od);
      r[g] = ((e & 0x0F0F0F0Fu) | (o & 0xF0F0F0F0u)) & pat;
    }
    *reinterpret_cast<uint4 *>(out + n * row_bytes + (pos >> 1)) = make_uint4(r[0], r[1], r[2], r[3]);
  }
}

}  // namespace

cudaError_t launch_pack_b_streams(const int16_t *code, int64_t N, int64_t ldk, int prec,
                                  int shift, bool e2m1, int64_t pool_period,
                                  const uint8_t *pool_comp, uint8_t *out, cudaStream_t s) {
  const int64_t total = N * ((ldk << prec) >> (e2m1 ? 5 : 4));
  if (total == 0) return cudaSuccess;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  if (e2m1)
    pack_b_streams_e2m1_kernel<<<(unsigned)blocks, 256, 0, s>>>(code, N, ldk, prec, shift,
                                                                pool_period, pool_comp, out);
  else
    pack_b_streams_kernel<<<(unsigned)blocks, 256, 0, s>>>(code, N, ldk, prec, shift,
                                                           pool_period, pool_comp, out);
  return cudaGetLastError();
}

bool launch_quantize_slices(const float *x, const GroupShape &g, int64_t K, int64_t ldc,
                            int mode, int prec, int16_t *code, float *rscale, int32_t *rzero,
                            int32_t *rsum, cudaStream_t s, cudaError_t *err) {
  // per-slice groups of whole slices, rows of 4 R fp32 values (R | 32),
  // unpadded code rows, 16-byte aligned slices that fit the registers
  const bool whole = g.group_rows == g.slice_rows && g.rows % g.slice_rows == 0;
  const int64_t R = K / 4;
  if (!whole || K % 4 != 0 || ldc != K || (R != 4 && R != 8 && R != 16 && R != 32) ||
      g.slice_rows * R > 256 * kSliceVec || (reinterpret_cast<uintptr_t>(x) & 15) != 0 ||
      g.ngroups > 0x7FFFFFFF)
    return false;
  *err = cudaSuccess;
  if (g.ngroups == 0) return true;
  const unsigned grid = (unsigned)g.ngroups;
  if (R == 4)
    quantize_slices_kernel<4><<<grid, 256, 0, s>>>(x, g.slice_rows, mode, prec, code, rscale,
                                                   rzero, rsum);
  else if (R == 8)
    quantize_slices_kernel<8><<<grid, 256, 0, s>>>(x, g.slice_rows, mode, prec, code, rscale,
                                                   rzero, rsum);
  else if (R == 16)
    quantize_slices_kernel<16><<<grid, 256, 0, s>>>(x, g.slice_rows, mode, prec, code, rscale,
                                                    rzero, rsum);
  else
    quantize_slices_kernel<32><<<grid, 256, 0, s>>>(x, g.slice_rows, mode, prec, code, rscale,
                                                    rzero, rsum);
  *err = cudaGetLastError();
  return true;
}

cudaError_t launch_softmax_quantize(const float *x, int64_t rows, int K, float scale, int mode,
                                    int prec, int64_t ldc, int16_t *code, float *rscale,
                                    int32_t *rzero, int32_t *rsum, float *probs, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  int64_t blocks = (rows + 7) / 8;  // 8 warps per block, one row per warp
  if (blocks > 148 * 16) blocks = 148 * 16;
#define SCMP_SOFTMAX_Q(NI)                                                                      \
  softmax_quantize_kernel<NI><<<(unsigned)blocks, 256, 0, s>>>(x, rows, K, scale, mode, prec, ldc, \
                                                               code, rscale, rzero, rsum, probs)
  // NI = ceil(K / 32) would do for the arithmetic: the elements torch's
  // kernel holds past that (up to the next power of two) are -inf, whose e =
  // +0 leaves the lane sums unchanged; 9 covers 257-token rows
  if (K <= 64)
    SCMP_SOFTMAX_Q(2);
  else if (K <= 128)
    SCMP_SOFTMAX_Q(4);
  else if (K <= 256)
    SCMP_SOFTMAX_Q(8);
  else if (K <= 288)
    SCMP_SOFTMAX_Q(9);
  else if (K <= 512)
    SCMP_SOFTMAX_Q(16);
  else
    SCMP_SOFTMAX_Q(32);
#undef SCMP_SOFTMAX_Q
  return cudaGetLastError();
}

cudaError_t launch_row_stats(const void *x, bool x_bf16, int64_t rows, int64_t K, int mode,
                             float2 *stat, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  const int threads = 256;
  // short rows (K <= 128): 8 lanes per row, 4 rows per warp
  const int lpr = K <= 128 ? 8 : 32;
  const int64_t blocks = (rows * lpr + threads - 1) / threads;
  const auto *xb = static_cast<const __nv_bfloat16 *>(x);
  const auto *xf = static_cast<const float *>(x);
  if (x_bf16 && lpr == 8)
    row_stats_kernel<__nv_bfloat16, 8><<<(unsigned)blocks, threads, 0, s>>>(xb, rows, K, mode, stat);
  else if (x_bf16)
    row_stats_kernel<__nv_bfloat16, 32><<<(unsigned)blocks, threads, 0, s>>>(xb, rows, K, mode,
                                                                             stat);
  else if (lpr == 8)
    row_stats_kernel<float, 8><<<(unsigned)blocks, threads, 0, s>>>(xf, rows, K, mode, stat);
  else
    row_stats_kernel<float, 32><<<(unsigned)blocks, threads, 0, s>>>(xf, rows, K, mode, stat);
  return cudaGetLastError();
}

cudaError_t launch_group_stats(const float2 *stat, const GroupShape &g, int mode, int prec,
                               float *gscale, float *ginv, int32_t *gzero, cudaStream_t s) {
  if (g.ngroups == 0) return cudaSuccess;
  if (g.group_rows <= 64) {
    const int64_t blocks = (g.ngroups + 255) / 256;
    group_stats_small_kernel<<<(unsigned)(blocks < 148 * 16 ? blocks : 148 * 16), 256, 0, s>>>(
        stat, g, mode, prec, gscale, ginv, gzero);
    return cudaGetLastError();
  }
  // few large groups (per-tensor / per-head over a whole batch): one wide
  // block per group keeps many row-stat loads in flight
  const int threads = g.ngroups < 296 ? 1024 : 256;
  group_stats_kernel<<<(unsigned)g.ngroups, threads, 0, s>>>(stat, g, mode, prec, gscale, ginv,
                                                             gzero);
  return cudaGetLastError();
}

cudaError_t launch_quantize(const void *x, bool x_bf16, const GroupShape &g, int64_t K,
                            int64_t ldc, int mode, int prec,
                            const float *gscale, const float *ginv, const int32_t *gzero,
                            int16_t *code, float *rscale, int32_t *rzero, int32_t *rsum,
                            cudaStream_t s) {
  if (g.rows == 0) return cudaSuccess;
  const int threads = 256;
  const int lpr = ldc <= 128 ? 8 : 32;  // short rows: 8 lanes per row
  const int64_t blocks = (g.rows * lpr + threads - 1) / threads;
  const auto *xb = static_cast<const __nv_bfloat16 *>(x);
  const auto *xf = static_cast<const float *>(x);
#define SCMP_QUANTIZE(T, LPR, X)                                                              \
  quantize_kernel<T, LPR><<<(unsigned)blocks, threads, 0, s>>>(X, g, K, ldc, mode, prec, gscale, \
                                                               ginv, gzero, code, rscale, rzero,  \
                                                               rsum)
  if (x_bf16 && lpr == 8)
    SCMP_QUANTIZE(__nv_bfloat16, 8, xb);
  else if (x_bf16)
    SCMP_QUANTIZE(__nv_bfloat16, 32, xb);
  else if (lpr == 8)
    SCMP_QUANTIZE(float, 8, xf);
  else
    SCMP_QUANTIZE(float, 32, xf);
#undef SCMP_QUANTIZE
  return cudaGetLastError();
}

cudaError_t launch_quantize_rows(const void *x, bool x_bf16, int64_t rows, int64_t K,
                                 int64_t ldc, int mode, int prec, int16_t *code, float *rscale,
                                 int32_t *rzero, int32_t *rsum, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  const int threads = 256;
  const int lpr = ldc <= 128 ? 8 : 32;  // short rows: 8 lanes per row
  const int64_t blocks = (rows * lpr + threads - 1) / threads;
  const auto *xb = static_cast<const __nv_bfloat16 *>(x);
  const auto *xf = static_cast<const float *>(x);
#define SCMP_QUANTIZE_ROWS(T, LPR, X)                                                        \
  quantize_rows_kernel<T, LPR><<<(unsigned)blocks, threads, 0, s>>>(X, rows, K, ldc, mode, prec, \
                                                                    code, rscale, rzero, rsum)
  if (x_bf16 && lpr == 8)
    SCMP_QUANTIZE_ROWS(__nv_bfloat16, 8, xb);
  else if (x_bf16)
    SCMP_QUANTIZE_ROWS(__nv_bfloat16, 32, xb);
  else if (lpr == 8)
    SCMP_QUANTIZE_ROWS(float, 8, xf);
  else
    SCMP_QUANTIZE_ROWS(float, 32, xf);
#undef SCMP_QUANTIZE_ROWS
  return cudaGetLastError();
}

cudaError_t launch_stream_table(const uint8_t *pool, int pool_dims, int prec, uint32_t *table,
                                uint2 *strips, cudaStream_t s) {
  const int T = 1 << prec;
  const int64_t threads = (int64_t)pool_dims * (T + 1) * (T >= 32 ? T / 32 : 1);
  const int64_t blocks = (threads + 255) / 256;
  stream_table_kernel<<<(unsigned)(blocks < 1184 ? blocks : 1184), 256, 0, s>>>(
      pool, pool_dims, prec, table, strips);
  return cudaGetLastError();
}

cudaError_t launch_pool_complement(const uint8_t *pool, int pool_dims, int64_t rows, int prec,
                                   int lp_log2, int shift, bool nibble_pairs, uint8_t *out,
                                   cudaStream_t s) {
  if (rows < pool_dims) rows = pool_dims;
  const int64_t bytes = rows << lp_log2;
  const int64_t blocks = (bytes + 255) / 256;
  pool_complement_kernel<<<(unsigned)(blocks < 296 ? blocks : 296), 256, 0, s>>>(
      pool, pool_dims, rows, prec, lp_log2, shift, nibble_pairs ? 1 : 0, out);
  return cudaGetLastError();
}

}  // namespace scmp
