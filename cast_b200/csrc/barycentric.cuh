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

namespace castk {

// ---------------------------------------------------------------------------
// The lift's control-conditioned weights (proposed/matrix_curvature_phase_
// frame_weave.py:3903-3951 control state, :4094-4194 weights): for target t
// between anchors l < r of its segment, with alpha = (t - l) / (r - l),
//   w = softmax([log1p(-alpha), log(alpha)] - lp * (1 - cos_cam) - la * (1 - cos_act))
// where cam(f) = normalize(mean over the frame's S spatial rows of the
// Plucker camera features) and act(f) = normalize(mouse | keyboard controls
// area-pooled from frame rate to latent cells, the memory frames' own
// controls for f < memory_frames), cosines clamped to [-1, 1].
// grid (N targets, B), 128 threads: each CTA pools its three frames.
// ---------------------------------------------------------------------------
constexpr int kLiftThreads = 128;
constexpr int kLiftMaxFeat = 16;   // Plucker features per row
constexpr int kLiftMaxAct = 64;    // mouse + keyboard channels
constexpr int kLiftMaxTargets = 64;

struct LiftCond {              // one control sequence [B, L, C] fp32, or null
  const float *x;
  int L, C;
};

struct LiftParams {
  const void *plucker;          // [B, rows >= T*S, P], fp32 or bf16
  int plucker_bf16, P, S, T, M, rows;
  LiftCond cur[2], mem[2];      // the given sequences in order (mouse, keyboard)
  int action;                   // any current control given
  float lp, la;
  float *weights;               // [B, N, 2]
  int N;
  int targets[kLiftMaxTargets][3];  // target, left, right frames
  int slots[kLiftMaxTargets][2];    // left, right anchor slots (rows of the active residual)
  int32_t *pairs_out;               // [N][2] slots for the pair writer, or null
  int32_t *frames_out;              // [N] target frames for the pair writer, or null
  float prior[kLiftMaxTargets][2];  // log1p(-alpha), log(alpha)
};

__device__ __forceinline__ float lift_plucker(const LiftParams &p, size_t i) {
  return p.plucker_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16 *>(p.plucker)[i])
                        : static_cast<const float *>(p.plucker)[i];
}

// adaptive_avg_pool1d's cell `cell` of `n` over the L frame-rate rows of one
// channel: rows [floor(cell*L/n), ceil((cell+1)*L/n))
__device__ __forceinline__ float lift_pool(const LiftCond &c, int b, int cell, int n, int ch) {
  if (c.L == n) return c.x[((size_t)b * c.L + cell) * c.C + ch];
  const int lo = (cell * c.L) / n, hi = ((cell + 1) * c.L + n - 1) / n;
  float s = 0.f;
  for (int r = lo; r < hi; ++r) s += c.x[((size_t)b * c.L + r) * c.C + ch];
  return s / (float)(hi - lo);
}

__global__ void __launch_bounds__(kLiftThreads) barycentric_weights_kernel(const __grid_constant__ LiftParams p) {
  __shared__ float cam[3][kLiftMaxFeat];
  __shared__ float act[3][kLiftMaxAct];
  __shared__ float red[kLiftThreads / 32][kLiftMaxFeat];
  const int n = blockIdx.x, b = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int fr[3];
  for (int j = 0; j < 3; ++j) fr[j] = p.targets[n][j];
  // camera: spatial mean of each frame's Plucker rows, then L2-normalised
  for (int j = 0; j < 3; ++j) {
    float acc[kLiftMaxFeat];
#pragma unroll
    for (int q = 0; q < kLiftMaxFeat; ++q) acc[q] = 0.f;
    for (int s = threadIdx.x; s < p.S; s += blockDim.x) {
      const size_t row = ((size_t)b * p.rows + (size_t)fr[j] * p.S + s) * p.P;
      for (int q = 0; q < p.P; ++q) acc[q] += lift_plucker(p, row + q);
    }
    for (int q = 0; q < p.P; ++q) {
      float v = acc[q];
      for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) red[warp][q] = v;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float nrm = 0.f;
      for (int q = 0; q < p.P; ++q) {
        float v = 0.f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) v += red[w][q];
        cam[j][q] = v / (float)p.S;
        nrm += cam[j][q] * cam[j][q];
      }
      const float inv = 1.f / fmaxf(sqrtf(nrm), 1e-8f);
      for (int q = 0; q < p.P; ++q) cam[j][q] *= inv;
    }
    __syncthreads();
  }
  // action: each frame's pooled controls, the given sequences concatenated
  // along channels in order (slot 0 then slot 1), normalised
  int A = 0;
  if (p.action) {
    A = (p.cur[0].x ? p.cur[0].C : 0) + (p.cur[1].x ? p.cur[1].C : 0);
    for (int i = threadIdx.x; i < 3 * A; i += blockDim.x) {
      const int j = i / A, ch = i % A;
      const bool memory = fr[j] < p.M;
      const int cell = memory ? fr[j] : fr[j] - p.M, cells = memory ? p.M : p.T - p.M;
      const LiftCond &s0 = memory ? p.mem[0] : p.cur[0], &s1 = memory ? p.mem[1] : p.cur[1];
      const int split = s0.x ? s0.C : 0;
      float v = 0.f;  // missing memory controls count as zeros
      if (ch < split) {
        v = lift_pool(s0, b, cell, cells, ch);
      } else if (s1.x) {
        v = lift_pool(s1, b, cell, cells, ch - split);
      }
      act[j][ch] = v;
    }
    __syncthreads();
    if (threadIdx.x < 3) {
      const int j = threadIdx.x;
      float nrm = 0.f;
      for (int ch = 0; ch < A; ++ch) nrm += act[j][ch] * act[j][ch];
      const float inv = 1.f / fmaxf(sqrtf(nrm), 1e-8f);
      for (int ch = 0; ch < A; ++ch) act[j][ch] *= inv;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    float logit[2];
    for (int side = 0; side < 2; ++side) {
      float cc = 0.f, ca = 0.f;
      for (int q = 0; q < p.P; ++q) cc += cam[0][q] * cam[1 + side][q];
      for (int ch = 0; ch < A; ++ch) ca += act[0][ch] * act[1 + side][ch];
      const float dc = 1.f - fminf(fmaxf(cc, -1.f), 1.f);
      const float da = 1.f - fminf(fmaxf(ca, -1.f), 1.f);  // no controls: 1 on both sides
      logit[side] = p.prior[n][side] - p.lp * dc - p.la * da;
    }
    const float mx = fmaxf(logit[0], logit[1]);
    const float e0 = expf(logit[0] - mx), e1 = expf(logit[1] - mx);
    const float sum = e0 + e1;
    p.weights[((size_t)b * p.N + n) * 2] = e0 / sum;
    p.weights[((size_t)b * p.N + n) * 2 + 1] = e1 / sum;
    if (b == 0 && p.pairs_out) {
      p.pairs_out[2 * n] = p.slots[n][0];
      p.pairs_out[2 * n + 1] = p.slots[n][1];
      p.frames_out[n] = p.targets[n][0];
    }
  }
}

}  // namespace castk
