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

// grid (chunks, targets): blockIdx.y is the target row, the x blocks stride
// over the frame's S*C values four at a time (16-byte loads and stores when
// the frame size is a multiple of 4, else one value at a time).  A slot or
// frame index out of range skips the row and is reported in the device error
// word.
__global__ void __launch_bounds__(kBaryThreads)
    barycentric_pair_kernel(const float *__restrict__ active, const float *__restrict__ weights,
                            const int32_t *__restrict__ pairs, const int32_t *__restrict__ targets,
                            float *__restrict__ out, long long sc, int A, int T, int mode) {
  const int n = blockIdx.y;
  const int ls = __ldg(&pairs[2 * n]), rs = __ldg(&pairs[2 * n + 1]);
  const int tf = __ldg(&targets[n]);
  if (ls < 0 || ls >= A || rs < 0 || rs >= A || tf < 0 || tf >= T) {
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(&g_cast_device_error, (int)CAST_ERR_INVALID_ARGUMENT);
    return;
  }
  const float wl = __ldg(&weights[2 * n]), wr = __ldg(&weights[2 * n + 1]);
  const float *left = active + (size_t)ls * sc;
  const float *right = active + (size_t)rs * sc;
  float *dst = out + (size_t)tf * sc;
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long first = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if ((sc & 3) == 0) {
    for (long long i = first; i < sc / 4; i += stride) {
      const float4 a = __ldg(reinterpret_cast<const float4 *>(left) + i);
      const float4 b = __ldg(reinterpret_cast<const float4 *>(right) + i);
      float4 o;
      o.x = bary_mix(mode, a.x, wl, b.x, wr);
      o.y = bary_mix(mode, a.y, wl, b.y, wr);
      o.z = bary_mix(mode, a.z, wl, b.z, wr);
      o.w = bary_mix(mode, a.w, wl, b.w, wr);
      reinterpret_cast<float4 *>(dst)[i] = o;
    }
  } else {
    for (long long i = first; i < sc; i += stride)
      dst[i] = bary_mix(mode, __ldg(left + i), wl, __ldg(right + i), wr);
  }
}

}  // namespace castk
