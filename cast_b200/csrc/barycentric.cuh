// Two-anchor residual writer of the control-barycentric reconstruction.
//
// For each target row n: out[target[n]] = mix(active[pair[n][0]] * w[n][0],
// active[pair[n][1]] * w[n][1]) over the S*C values of a frame, the weights
// computed by the caller.  Replaces the reference's direct pair writer
// (proposed/matrix_control_barycentric_pair_kernel.py:22-112), called from the
// frame weave's control-barycentric lift (proposed/matrix_curvature_phase_
// frame_weave.py:4278-4286).  An HBM copy: two frames read, one written.
#pragma once

#include "common.cuh"

namespace castk {

constexpr int kBaryThreads = 256;

// Rounding of the mix, as the reference's arithmetic modes state it:
//   1 separate:            RN(RN(l*wl) + RN(r*wr))
//   2 left_then_right_fma: FMA(r, wr, RN(l*wl))
//   3 right_then_left_fma: FMA(l, wl, RN(r*wr))
__device__ __forceinline__ float bary_mix(int mode, float l, float wl, float r, float wr) {
  if (mode == 1) return __fadd_rn(__fmul_rn(l, wl), __fmul_rn(r, wr));
  if (mode == 3) return __fmaf_rn(l, wl, __fmul_rn(r, wr));
  return __fmaf_rn(r, wr, __fmul_rn(l, wl));
}

// One grid over the frame's S*C values, four at a time (16-byte loads and
// stores when the frame size is a multiple of 4, else one value at a time);
// each thread writes its values for every target row in turn, so target rows
// that share anchor frames (targets between the same two anchors) read them
// from L1/L2 instead of HBM.  A row whose slots or frame are out of range is
// skipped and reported in the device error word.
__global__ void __launch_bounds__(kBaryThreads)
    barycentric_pair_kernel(const float *__restrict__ active, const float *__restrict__ weights,
                            const int32_t *__restrict__ pairs, const int32_t *__restrict__ targets,
                            float *__restrict__ out, long long sc, int A, int T, int N, int mode) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long first = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const bool vec = (sc & 3) == 0;
  for (int n = 0; n < N; ++n) {
    const int ls = __ldg(&pairs[2 * n]), rs = __ldg(&pairs[2 * n + 1]);
    const int tf = __ldg(&targets[n]);
    if (ls < 0 || ls >= A || rs < 0 || rs >= A || tf < 0 || tf >= T) {
      if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(&g_cast_device_error, (int)CAST_ERR_INVALID_ARGUMENT);
      continue;
    }
    const float wl = __ldg(&weights[2 * n]), wr = __ldg(&weights[2 * n + 1]);
    const float *left = active + (size_t)ls * sc;
    const float *right = active + (size_t)rs * sc;
    float *dst = out + (size_t)tf * sc;
    if (vec) {
      // four 16-byte loads of each anchor in flight per thread
      const long long n4 = sc / 4;
      for (long long i0 = first; i0 < n4; i0 += 4 * stride) {
        float4 a[4], b[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const long long i = i0 + u * stride;
          if (i < n4) {
            a[u] = __ldg(reinterpret_cast<const float4 *>(left) + i);
            b[u] = __ldg(reinterpret_cast<const float4 *>(right) + i);
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const long long i = i0 + u * stride;
          if (i < n4) {
            float4 o;
            o.x = bary_mix(mode, a[u].x, wl, b[u].x, wr);
            o.y = bary_mix(mode, a[u].y, wl, b[u].y, wr);
            o.z = bary_mix(mode, a[u].z, wl, b[u].z, wr);
            o.w = bary_mix(mode, a[u].w, wl, b[u].w, wr);
            reinterpret_cast<float4 *>(dst)[i] = o;
          }
        }
      }
    } else {
      for (long long i = first; i < sc; i += stride)
        dst[i] = bary_mix(mode, __ldg(left + i), wl, __ldg(right + i), wr);
    }
  }
}

}  // namespace castk
