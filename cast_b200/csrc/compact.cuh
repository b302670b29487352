// Compact-layout packing for the compact selection / attention path, with
// the RoPE phase applied on the way.
//
// The reference prepares each compact layer call with a chain of PyTorch
// ops: q and k rotated by the per-token RoPE phase in fp32
// (proposed/matrix_curvature_phase_frame_weave.py:5565-5574), then q, k and
// v gathered into packed blocks, transposed to [B,H,P,D] and zeroed at the
// padding slots (:5677-5684), cast to bf16 by the attention launch, and the
// attention output scattered back to token order (:6095).  Here one kernel
// does the rotation, gather, transpose, zeroing and cast in a single pass
// over q, k and v, and one kernel does the scatter: both are HBM copies.
#pragma once

#include "common.cuh"

namespace castk {

constexpr int kCompactThreads = 128;
constexpr int kCompactD = 128;  // head dim of the compact path

__device__ __forceinline__ void load8(const __nv_bfloat16 *p, float (&x)[8]) {
  const uint4 w = *reinterpret_cast<const uint4 *>(p);
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[2 * i] = __uint_as_float(u[i] << 16);
    x[2 * i + 1] = __uint_as_float(u[i] & 0xFFFF0000u);
  }
}
__device__ __forceinline__ void load8(const float *p, float (&x)[8]) {
  const float4 a = *reinterpret_cast<const float4 *>(p);
  const float4 b = *reinterpret_cast<const float4 *>(p + 4);
  x[0] = a.x, x[1] = a.y, x[2] = a.z, x[3] = a.w;
  x[4] = b.x, x[5] = b.y, x[6] = b.z, x[7] = b.w;
}
__device__ __forceinline__ uint4 to_bf16x8(const float (&x)[8]) {
  uint32_t u[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
    u[i] = *reinterpret_cast<const uint32_t *>(&h);
  }
  return make_uint4(u[0], u[1], u[2], u[3]);
}

// One CTA per packed row (b, p), grid-strided.  The row's token slab [H, D]
// is contiguous in q, k and v ([B,L,H,D]); each thread takes 8 consecutive
// values of one head (16 threads per head), rotates q and k by the phase
// ((a + ib)(c + is) with every product and sum rounded in fp32, no fused
// multiply-add, as the reference's complex64 multiply), rounds to bf16 and
// writes 16 bytes to [b, h, p, :].  Padding slots (index < 0) are written as
// zeros; an index >= L is treated the same and flagged in err.
template <typename InT>
__global__ void __launch_bounds__(kCompactThreads)
    compact_pack_kernel(const InT *__restrict__ q, const InT *__restrict__ k,
                        const InT *__restrict__ v, const float2 *__restrict__ phase,
                        int phase_heads, const int32_t *__restrict__ block_indices, int B, int L,
                        int H, int P, __nv_bfloat16 *__restrict__ qo, __nv_bfloat16 *__restrict__ ko,
                        __nv_bfloat16 *__restrict__ vo) {
  int *err = &g_cast_device_error;
  const int chunks = H * (kCompactD / 8);
  for (long long row = blockIdx.x; row < (long long)B * P; row += gridDim.x) {
    const int b = (int)(row / P), p = (int)(row % P);
    int t = __ldg(&block_indices[p]);
    if (t >= L) {
      if (threadIdx.x == 0) atomicExch(err, (int)CAST_ERR_INVALID_ARGUMENT);
      t = -1;
    }
    for (int c = threadIdx.x; c < chunks; c += blockDim.x) {
      const int h = c / (kCompactD / 8);
      const int j0 = (c % (kCompactD / 8)) * 8;
      const size_t dst = (((size_t)b * H + h) * P + p) * kCompactD + j0;
      if (t < 0) {
        const uint4 z = make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4 *>(qo + dst) = z;
        *reinterpret_cast<uint4 *>(ko + dst) = z;
        *reinterpret_cast<uint4 *>(vo + dst) = z;
        continue;
      }
      const size_t src = (((size_t)b * L + t) * H + h) * kCompactD + j0;
      float xq[8], xk[8], xv[8];
      load8(q + src, xq);
      load8(k + src, xk);
      load8(v + src, xv);
      if (phase) {
        const float4 *ph = reinterpret_cast<const float4 *>(
            phase + (((size_t)t * phase_heads + (phase_heads > 1 ? h : 0)) * (kCompactD / 2) + j0 / 2));
        const float4 p01 = __ldg(ph), p23 = __ldg(ph + 1);
        const float cs[8] = {p01.x, p01.y, p01.z, p01.w, p23.x, p23.y, p23.z, p23.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float c_ = cs[2 * i], s_ = cs[2 * i + 1];
          float a = xq[2 * i], bb = xq[2 * i + 1];
          xq[2 * i] = __fsub_rn(__fmul_rn(a, c_), __fmul_rn(bb, s_));
          xq[2 * i + 1] = __fadd_rn(__fmul_rn(a, s_), __fmul_rn(bb, c_));
          a = xk[2 * i], bb = xk[2 * i + 1];
          xk[2 * i] = __fsub_rn(__fmul_rn(a, c_), __fmul_rn(bb, s_));
          xk[2 * i + 1] = __fadd_rn(__fmul_rn(a, s_), __fmul_rn(bb, c_));
        }
      }
      *reinterpret_cast<uint4 *>(qo + dst) = to_bf16x8(xq);
      *reinterpret_cast<uint4 *>(ko + dst) = to_bf16x8(xk);
      *reinterpret_cast<uint4 *>(vo + dst) = to_bf16x8(xv);
    }
  }
}

// One CTA per token (b, t), grid-strided: out[b, t, h, :] = packed[b, h,
// token_to_packed[t], :] (the attention output back in token order).  A
// position outside [0, P) gives zeros and is flagged in err.
__global__ void __launch_bounds__(kCompactThreads)
    compact_unpack_kernel(const __nv_bfloat16 *__restrict__ packed,
                          const int32_t *__restrict__ token_to_packed, int B, int L, int H, int P,
                          __nv_bfloat16 *__restrict__ out) {
  int *err = &g_cast_device_error;
  const int chunks = H * (kCompactD / 8);
  for (long long row = blockIdx.x; row < (long long)B * L; row += gridDim.x) {
    const int b = (int)(row / L), t = (int)(row % L);
    const int pp = __ldg(&token_to_packed[t]);
    const bool ok = pp >= 0 && pp < P;
    if (!ok && threadIdx.x == 0) atomicExch(err, (int)CAST_ERR_INVALID_ARGUMENT);
    for (int c = threadIdx.x; c < chunks; c += blockDim.x) {
      const int h = c / (kCompactD / 8);
      const int j0 = (c % (kCompactD / 8)) * 8;
      uint4 w = make_uint4(0u, 0u, 0u, 0u);
      if (ok) w = *reinterpret_cast<const uint4 *>(packed + (((size_t)b * H + h) * P + pp) * kCompactD + j0);
      *reinterpret_cast<uint4 *>(out + (((size_t)b * L + t) * H + h) * kCompactD + j0) = w;
    }
  }
}

}  // namespace castk
