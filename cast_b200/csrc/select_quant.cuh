// Pooled-QK block scoring, top-k block selection and the per-block symmetric
// int8 quantiser (HBM-bound; one read of Q/K from HBM, the second pass of a
// block hits L2).
//
// Fixed arithmetic order (mirrored by the CPU oracle so that indices and
// codes compare bit-exactly):
//   * block sums: row r of a block accumulated into partial r % kSumLanes in
//     increasing r in float32 (IEEE adds from 0), partials widened to float64
//     and added in order 0..15;
//   * ||mean||^2 and every pooled dot product: lane l (of 32) sums the
//     products of dims d = l, l+32, ... in increasing d (multiply and add
//     rounded separately), then an xor-butterfly over 16, 8, 4, 2, 1;
//   * int8 code = clamp(rint_half_even(fl32(x / s)), -127, 127).
#pragma once

#include "common.cuh"

namespace castk {

constexpr int kSumLanes = 16;
constexpr double kNormEps = 1e-12;

__device__ __forceinline__ void bf16x8_to_f32(const uint4 &raw, float (&f)[8]) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// L2 cache policies: a block's statistics pass marks its lines evict-last so
// they survive until the quantisation pass re-reads them (evict-first there,
// and for the codes, which are not re-read by this kernel).
__device__ __forceinline__ uint64_t l2_evict_last() {
  uint64_t p;
  asm("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t p;
  asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint4 ldg_nc_v4_hint(const void *p, uint64_t pol) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p), "l"(pol));
  return r;
}
__device__ __forceinline__ uint4 ldg_v4_hint(const void *p, uint64_t pol) {
  uint4 r;
  asm volatile("ld.global.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p), "l"(pol));
  return r;
}
__device__ __forceinline__ void stg_v2_hint(void *p, uint2 v, uint64_t pol) {
  asm volatile("st.global.L2::cache_hint.v2.u32 [%0], {%1,%2}, %3;" ::"l"(p), "r"(v.x), "r"(v.y),
               "l"(pol)
               : "memory");
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// rint_half_even(fl32(x/s)) clamped to [-127,127], bit-exact with IEEE
// division.  Fast path: x * (1/s); when that quotient lies within 1e-4 of a
// half-integer (where the rounded product could round differently from the
// correctly rounded quotient) the exact IEEE division is used instead.
__device__ __forceinline__ int quant_code(float x, float s, float inv_s) {
  const float kMagic = 12582912.0f;  // 1.5 * 2^23
  float qv = __fmul_rn(x, inv_s);
  float t = __fadd_rn(qv, kMagic);
  float r = __fsub_rn(t, kMagic);
  if (fabsf(__fsub_rn(qv, r)) > 0.4999f) {
    qv = __fdiv_rn(x, s);
    t = __fadd_rn(qv, kMagic);
  }
  int c = __float_as_int(t) - 0x4B400000;
  return max(-127, min(127, c));
}

// Packed f32x2 helpers (two fp32 lanes per instruction, IEEE round-to-nearest).
__device__ __forceinline__ uint64_t q2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ uint64_t q2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t q2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t q2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// Codes of 8 values as 8 bytes, equal to quant_code() for every input of a
// block with amax >= 2^-90:  q0 = RN(x * inv), r = x - q0*s (exact, FMA),
// q1 = RN(q0 + r*inv) is the correctly rounded x/s (Markstein's correction
// step with inv = RN(1/s)); rint(q1) comes from the 1.5*2^23 shift, whose low
// byte is the code (|x| <= amax keeps |code| <= 127, so nothing is clamped).
// Checked against IEEE division for every bf16 amax and every bf16 x with
// |x| <= amax (tests/quant_fastpath_exhaustive.c); blocks with amax < 2^-90,
// where the residual could be subnormal, use quant_code().
__device__ __forceinline__ uint2 quant8_fast(const float (&f)[8], uint64_t invx2, uint64_t negsx2) {
  const uint64_t magic = q2_pack(12582912.0f, 12582912.0f);
  uint32_t t[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint64_t x = q2_pack(f[2 * i], f[2 * i + 1]);
    const uint64_t q0 = q2_mul(x, invx2);
    const uint64_t r = q2_fma(q0, negsx2, x);
    const uint64_t tt = q2_add(q2_fma(r, invx2, q0), magic);
    t[2 * i] = (uint32_t)tt;
    t[2 * i + 1] = (uint32_t)(tt >> 32);
  }
  const uint32_t lo = __byte_perm(__byte_perm(t[0], t[1], 0x0040), __byte_perm(t[2], t[3], 0x0040), 0x5410);
  const uint32_t hi = __byte_perm(__byte_perm(t[4], t[5], 0x0040), __byte_perm(t[6], t[7], 0x0040), 0x5410);
  return make_uint2(lo, hi);
}

__device__ __forceinline__ float quant_scale_of(float amax) {
  return amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
}

// Lane-partial + butterfly sum of a[d]*b[d] over D dims (warp-collective).
template <int D>
__device__ __forceinline__ double warp_dot(const double *a, const double *b, int lane) {
  double part = __dmul_rn(a[lane], b[lane]);
#pragma unroll
  for (int d = lane + 32; d < D; d += 32) part = __dadd_rn(part, __dmul_rn(a[d], b[d]));
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) part = __dadd_rn(part, __shfl_xor_sync(0xffffffffu, part, s));
  return part;
}

// The int8 codes of one block (second pass): each thread takes rows slot,
// slot + 16, ... of its 8-column group; `fast` selects the division-free
// path (exact for blocks with amax >= 2^-90), else the IEEE division;
// padding rows (vrow[r] == 0) get code 0.
template <int D, bool kMasked>
__device__ __forceinline__ void write_block_codes(const __nv_bfloat16 *base, int8_t *cbase, int rows,
                                                  int slot, const uint8_t *vrow, float sc, bool fast,
                                                  uint64_t drop_pol) {
  constexpr int kUnroll = 8;
  const float inv = __frcp_rn(sc);
  const uint64_t invx2 = q2_pack(inv, inv), negsx2 = q2_pack(-sc, -sc);
  auto quant8 = [&](const uint4 &raw) {
    float f[8];
    bf16x8_to_f32(raw, f);
    if (fast) return quant8_fast(f, invx2, negsx2);
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) lo |= (uint32_t)(quant_code(f[i], sc, inv) & 0xFF) << (8 * i);
#pragma unroll
    for (int i = 0; i < 4; ++i) hi |= (uint32_t)(quant_code(f[4 + i], sc, inv) & 0xFF) << (8 * i);
    return make_uint2(lo, hi);
  };
  int rr = slot;
  for (; rr + (kUnroll - 1) * kSumLanes < rows; rr += kUnroll * kSumLanes) {
    uint4 raw[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
      raw[u] = ldg_v4_hint(base + (size_t)(rr + u * kSumLanes) * D, drop_pol);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      uint2 c = quant8(raw[u]);
      if (kMasked && vrow && !vrow[rr + u * kSumLanes]) c = make_uint2(0u, 0u);
      stg_v2_hint(cbase + (size_t)(rr + u * kSumLanes) * D, c, drop_pol);
    }
  }
  for (; rr < rows; rr += kSumLanes) {
    uint2 c = quant8(ldg_v4_hint(base + (size_t)rr * D, drop_pol));
    if (kMasked && vrow && !vrow[rr]) c = make_uint2(0u, 0u);
    stg_v2_hint(cbase + (size_t)rr * D, c, drop_pol);
  }
}

// ---------------------------------------------------------------------------
// Kernel 1: per-(bh, block) pooled statistics and int8 codes.
// grid.x spans [Q blocks | K blocks | V blocks], grid.y = B*H.
// Threads: 16 row slots x D/8 column groups (8 bf16 = 16 bytes each).
// ---------------------------------------------------------------------------
// kMasked: q_valid / k_valid may be given (token validity of the compact
// packing; k_valid also covers V).  An invalid token's row is read and
// replaced by zeros -- exactly the restatement's zero-padded sums -- leaves
// the block's pooled-mean denominator and RMS count, and gets code 0.
template <int D, bool kMasked>
__global__ void __launch_bounds__(kSumLanes *(D / 8), 4)
    pool_quant_kernel(const __nv_bfloat16 *__restrict__ q, const __nv_bfloat16 *__restrict__ k,
                      const __nv_bfloat16 *__restrict__ v, const uint8_t *__restrict__ q_valid,
                      const uint8_t *__restrict__ k_valid, int Lq, int Lk, int block, int nqb,
                      int nkb, int8_t *q_codes, float *q_scales, int8_t *k_codes,
                      float *k_scales, int8_t *v_codes, float *v_scales, double *pooled,
                      float *block_rms, uint8_t *need_flags) {
  constexpr int kGroups = D / 8;
  constexpr int kThreads = kSumLanes * kGroups;
  __shared__ float red[kSumLanes][D];
  __shared__ double mean_s[D];
  __shared__ float wmax[kThreads / 32];
  __shared__ float wsq[kThreads / 32];
  __shared__ float s_scale;
  __shared__ float s_amax;
  __shared__ double s_denom;
  __shared__ int s_count;  // valid rows of the block

  const int tid = threadIdx.x;
  const int grp = tid % kGroups;
  const int slot = tid / kGroups;
  const int bh = blockIdx.y;
  int blk = blockIdx.x;
  int which;  // 0 = Q, 1 = K, 2 = V
  if (blk < nqb) {
    which = 0;
  } else if (blk < nqb + nkb) {
    which = 1;
    blk -= nqb;
  } else {
    which = 2;
    blk -= nqb + nkb;
  }
  const __nv_bfloat16 *X = which == 0 ? q : (which == 1 ? k : v);
  const int L = which == 0 ? Lq : Lk;
  int8_t *codes = which == 0 ? q_codes : (which == 1 ? k_codes : v_codes);
  float *scales = which == 0 ? q_scales : (which == 1 ? k_scales : v_scales);
  const int nb = which == 0 ? nqb : nkb;

  const int b0 = blk * block;
  const int rows = min(block, L - b0);
  const __nv_bfloat16 *base = X + ((size_t)bh * L + b0) * D + grp * 8;
  const uint8_t *vrow = kMasked ? (which == 0 ? q_valid : k_valid) : nullptr;  // may be null
  if (vrow) vrow += b0;
  if (tid == 0) s_count = kMasked && vrow ? 0 : rows;
  __syncthreads();
  int my_count = 0;  // valid rows among this thread's (column group 0 only)

  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
  float amax = 0.0f, sq = 0.0f;
  const bool pool = which != 2;

  constexpr int kUnroll = 8;
  const uint64_t keep_pol = l2_evict_last(), drop_pol = l2_evict_first();
  int r = slot;
  for (; r + (kUnroll - 1) * kSumLanes < rows; r += kUnroll * kSumLanes) {
    uint4 raw[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
      raw[u] = ldg_nc_v4_hint(base + (size_t)(r + u * kSumLanes) * D, keep_pol);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      float f[8];
      bf16x8_to_f32(raw[u], f);
      if (kMasked && vrow) {
        const bool ok = vrow[r + u * kSumLanes] != 0;
        my_count += ok;
#pragma unroll
        for (int i = 0; i < 8; ++i) f[i] = ok ? f[i] : 0.0f;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (pool) acc[i] = __fadd_rn(acc[i], f[i]);
        amax = fmaxf(amax, fabsf(f[i]));
        sq = fmaf(f[i], f[i], sq);
      }
    }
  }
  for (; r < rows; r += kSumLanes) {
    float f[8];
    bf16x8_to_f32(ldg_nc_v4_hint(base + (size_t)r * D, keep_pol), f);
    if (kMasked && vrow) {
      const bool ok = vrow[r] != 0;
      my_count += ok;
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] = ok ? f[i] : 0.0f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (pool) acc[i] = __fadd_rn(acc[i], f[i]);
      amax = fmaxf(amax, fabsf(f[i]));
      sq = fmaf(f[i], f[i], sq);
    }
  }

  // amax / sum of squares across the CTA (order-independent for amax).
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) {
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, s));
    sq += __shfl_xor_sync(0xffffffffu, sq, s);
  }
  if ((tid & 31) == 0) {
    wmax[tid >> 5] = amax;
    wsq[tid >> 5] = sq;
  }
  if (pool) {
#pragma unroll
    for (int i = 0; i < 8; ++i) red[slot][grp * 8 + i] = acc[i];
  }
  if (kMasked && vrow && grp == 0 && my_count) atomicAdd(&s_count, my_count);
  __syncthreads();
  const int count = s_count;
  if (tid == 0) {
    float m = 0.0f, s2 = 0.0f;
    for (int w = 0; w < kThreads / 32; ++w) {
      m = fmaxf(m, wmax[w]);
      s2 += wsq[w];
    }
    const float sc = quant_scale_of(m);
    s_scale = sc;
    s_amax = m;
    if (scales) scales[(size_t)bh * nb + blk] = sc;
    if (block_rms && pool) {
      const int row0 = which == 0 ? 0 : nqb;
      block_rms[(size_t)bh * (nqb + nkb) + row0 + blk] =
          sqrtf(s2 / (float)max(1, count * D));
    }
    // the block is not needed until an int8 query block marks it
    if (need_flags && pool) need_flags[(size_t)bh * (nqb + nkb) + (which == 0 ? 0 : nqb) + blk] = 0;
  }
  if (pool) {
    if (tid < D) {
      double t = (double)red[0][tid];
#pragma unroll
      for (int p = 1; p < kSumLanes; ++p) t = __dadd_rn(t, (double)red[p][tid]);
      mean_s[tid] = __ddiv_rn(t, (double)max(count, 1));
    }
    __syncthreads();
    if (tid < 32) {
      double part = __dmul_rn(mean_s[tid], mean_s[tid]);
#pragma unroll
      for (int d = tid + 32; d < D; d += 32) part = __dadd_rn(part, __dmul_rn(mean_s[d], mean_s[d]));
#pragma unroll
      for (int s = 16; s >= 1; s >>= 1) part = __dadd_rn(part, __shfl_xor_sync(0xffffffffu, part, s));
      if (tid == 0) s_denom = fmax(__dsqrt_rn(part), kNormEps);
    }
    __syncthreads();
    if (tid < D) {
      const int row0 = which == 0 ? 0 : nqb;
      pooled[((size_t)bh * (nqb + nkb) + row0 + blk) * D + tid] = __ddiv_rn(mean_s[tid], s_denom);
    }
  } else {
    __syncthreads();
  }

  // Second pass: int8 codes (the block was just read; these loads hit L2).
  if (codes)
    write_block_codes<D, kMasked>(base, codes + ((size_t)bh * L + b0) * D + grp * 8, rows, slot, vrow,
                                  s_scale, s_amax >= 0x1p-90f, drop_pol);
}

// Kernel 1s: kernel 1 for unmasked Q/K blocks that fit in shared memory,
// with the block staged there by bulk copies so the codes come from shared
// memory instead of a second read of the block: HBM sees the block once and
// the codes once.  The same threads take the same rows in the same order as
// kernel 1, so the sums, amax, RMS, pooled vectors and codes are bit-identical
// to it.  Dynamic shared memory: the block (rows x D bf16), reused for the
// row-slot partial sums after the codes are written.  One CTA per SM.
constexpr int kStageChunk = 32768;  // bytes per bulk copy

template <int D>
__global__ void __launch_bounds__(kSumLanes *(D / 8), 1)
    pool_quant_staged_kernel(const __nv_bfloat16 *__restrict__ q, const __nv_bfloat16 *__restrict__ k,
                             int Lq, int Lk, int block, int nqb, int nkb, int8_t *q_codes,
                             float *q_scales, int8_t *k_codes, float *k_scales, double *pooled,
                             float *block_rms) {
  constexpr int kGroups = D / 8;
  constexpr int kThreads = kSumLanes * kGroups;
  extern __shared__ __align__(128) unsigned char stage_raw[];
  __shared__ __align__(8) uint64_t full_bar;
  __shared__ int cta_abort;
  __shared__ double mean_s[D];
  __shared__ float wmax[kThreads / 32];
  __shared__ float wsq[kThreads / 32];
  __shared__ float s_scale;
  __shared__ float s_amax;
  __shared__ double s_denom;

  const int tid = threadIdx.x;
  const int grp = tid % kGroups;
  const int slot = tid / kGroups;
  const int bh = blockIdx.y;
  int blk = blockIdx.x;
  const bool is_q = blk < nqb;
  if (!is_q) blk -= nqb;
  const __nv_bfloat16 *X = is_q ? q : k;
  const int L = is_q ? Lq : Lk;
  int8_t *codes = is_q ? q_codes : k_codes;
  float *scales = is_q ? q_scales : k_scales;
  const int nb = is_q ? nqb : nkb;
  const int b0 = blk * block;
  const int rows = min(block, L - b0);
  const unsigned char *src = reinterpret_cast<const unsigned char *>(X + ((size_t)bh * L + b0) * D);
  const uint32_t bytes = (uint32_t)rows * D * 2;
  __nv_bfloat16 *st = reinterpret_cast<__nv_bfloat16 *>(stage_raw);

  if (tid == 0) {
    cta_abort = 0;
    castdev::mbar_init(&full_bar, 1);
    castdev::fence_barrier_init();
    castdev::mbar_arrive_expect_tx(&full_bar, bytes);
    for (uint32_t off = 0; off < bytes; off += kStageChunk)
      castdev::bulk_load(stage_raw + off, src + off, min((uint32_t)kStageChunk, bytes - off), &full_bar);
  }
  __syncthreads();
  // the copies always complete; a wait that gives up leaves the statistics
  // and codes of this block unwritten and sets the device error word
  const bool ok = castdev::mbar_wait_drain(&full_bar, 0, &cta_abort);

  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
  float amax = 0.0f, sq = 0.0f;
  const __nv_bfloat16 *base = st + grp * 8;
  if (ok) {
    for (int r = slot; r < rows; r += kSumLanes) {
      float f[8];
      bf16x8_to_f32(*reinterpret_cast<const uint4 *>(base + (size_t)r * D), f);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        acc[i] = __fadd_rn(acc[i], f[i]);
        amax = fmaxf(amax, fabsf(f[i]));
        sq = fmaf(f[i], f[i], sq);
      }
    }
  }
#pragma unroll
  for (int s2 = 16; s2 >= 1; s2 >>= 1) {
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, s2));
    sq += __shfl_xor_sync(0xffffffffu, sq, s2);
  }
  if ((tid & 31) == 0) {
    wmax[tid >> 5] = amax;
    wsq[tid >> 5] = sq;
  }
  __syncthreads();
  if (tid == 0) {
    float m = 0.0f, s2 = 0.0f;
    for (int w = 0; w < kThreads / 32; ++w) {
      m = fmaxf(m, wmax[w]);
      s2 += wsq[w];
    }
    const float sc = quant_scale_of(m);
    s_scale = sc;
    s_amax = m;
    if (ok) {
      scales[(size_t)bh * nb + blk] = sc;
      block_rms[(size_t)bh * (nqb + nkb) + (is_q ? 0 : nqb) + blk] = sqrtf(s2 / (float)max(1, rows * D));
    }
  }
  __syncthreads();
  // codes from the staged block
  if (ok && codes) {
    const float sc = s_scale;
    const bool fast = s_amax >= 0x1p-90f;
    const float inv = __frcp_rn(sc);
    const uint64_t invx2 = q2_pack(inv, inv), negsx2 = q2_pack(-sc, -sc);
    const uint64_t drop_pol = l2_evict_first();
    int8_t *cbase = codes + ((size_t)bh * L + b0) * D + grp * 8;
    for (int r = slot; r < rows; r += kSumLanes) {
      float f[8];
      bf16x8_to_f32(*reinterpret_cast<const uint4 *>(base + (size_t)r * D), f);
      uint2 c;
      if (fast) {
        c = quant8_fast(f, invx2, negsx2);
      } else {
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) lo |= (uint32_t)(quant_code(f[i], sc, inv) & 0xFF) << (8 * i);
#pragma unroll
        for (int i = 0; i < 4; ++i) hi |= (uint32_t)(quant_code(f[4 + i], sc, inv) & 0xFF) << (8 * i);
        c = make_uint2(lo, hi);
      }
      stg_v2_hint(cbase + (size_t)r * D, c, drop_pol);
    }
  }
  __syncthreads();  // the staged block is no longer read: its first bytes hold the partial sums
  float (*red)[D] = reinterpret_cast<float (*)[D]>(stage_raw);
#pragma unroll
  for (int i = 0; i < 8; ++i) red[slot][grp * 8 + i] = acc[i];
  __syncthreads();
  if (tid < D) {
    double t = (double)red[0][tid];
#pragma unroll
    for (int p = 1; p < kSumLanes; ++p) t = __dadd_rn(t, (double)red[p][tid]);
    mean_s[tid] = __ddiv_rn(t, (double)max(rows, 1));
  }
  __syncthreads();
  if (tid < 32) {
    double part = __dmul_rn(mean_s[tid], mean_s[tid]);
#pragma unroll
    for (int d = tid + 32; d < D; d += 32) part = __dadd_rn(part, __dmul_rn(mean_s[d], mean_s[d]));
#pragma unroll
    for (int s2 = 16; s2 >= 1; s2 >>= 1) part = __dadd_rn(part, __shfl_xor_sync(0xffffffffu, part, s2));
    if (tid == 0) s_denom = fmax(__dsqrt_rn(part), kNormEps);
  }
  __syncthreads();
  if (ok && tid < D)
    pooled[((size_t)bh * (nqb + nkb) + (is_q ? 0 : nqb) + blk) * D + tid] = __ddiv_rn(mean_s[tid], s_denom);
}

// Bytes of shared memory kernel 1s needs for a block (0: it does not fit).
constexpr size_t kStagedStaticBytes = 4096;  // mean_s, the reductions, the barrier
__host__ __device__ inline size_t staged_block_bytes(int block, int D) {
  const size_t b = (size_t)block * D * 2;
  if (block < 2 * kSumLanes) return 0;  // the partial sums reuse the buffer
  return b + kStagedStaticBytes <= 227 * 1024 ? b : 0;
}

// Kernel 3 (auto policy): int8 codes only for the blocks an int8 query block
// reads -- its own Q block and every K block it selected, which the
// selection kernel marked in need_flags ([B*H][nQb + nKb], cleared by kernel
// 1); the other code bytes are left as they are.  The grid strides over the
// flags (blocks in (bh, block) order; launched with one CTA per block, so
// an unmarked block's CTA exits after one byte) and codes the marked blocks
// with kernel 1's scale.  The division-free path is taken for
// scale >= 2^-96, which implies amax >= 127 * 2^-96 * (1 - 2^-24) > 2^-90
// (where it is exact); smaller blocks use the division, so the codes equal
// kernel 1's fused second pass bit for bit.
template <int D, bool kMasked>
__global__ void __launch_bounds__(kSumLanes *(D / 8), 4)
    quant_needed_kernel(const __nv_bfloat16 *__restrict__ q, const __nv_bfloat16 *__restrict__ k,
                        const uint8_t *__restrict__ q_valid, const uint8_t *__restrict__ k_valid,
                        int Lq, int Lk, int block, int nqb, int nkb, int BH,
                        const uint8_t *__restrict__ need_flags, int8_t *q_codes,
                        const float *__restrict__ q_scales, int8_t *k_codes,
                        const float *__restrict__ k_scales) {
  constexpr int kGroups = D / 8;
  const int tid = threadIdx.x;
  const int grp = tid % kGroups, slot = tid / kGroups;
  const int per = nqb + nkb;
  for (int id = blockIdx.x; id < BH * per; id += gridDim.x) {
    if (!need_flags[id]) continue;  // block-uniform
    const int bh = id / per, x = id % per;
    const bool is_q = x < nqb;
    const int blk = is_q ? x : x - nqb;
    const __nv_bfloat16 *X = is_q ? q : k;
    const int L = is_q ? Lq : Lk;
    const int b0 = blk * block;
    const int rows = min(block, L - b0);
    const uint8_t *vrow = kMasked ? (is_q ? q_valid : k_valid) : nullptr;
    if (vrow) vrow += b0;
    const float sc = is_q ? q_scales[(size_t)bh * nqb + blk] : k_scales[(size_t)bh * nkb + blk];
    int8_t *codes = is_q ? q_codes : k_codes;
    write_block_codes<D, kMasked>(X + ((size_t)bh * L + b0) * D + grp * 8,
                                  codes + ((size_t)bh * L + b0) * D + grp * 8, rows, slot, vrow, sc,
                                  sc >= 0x1p-96f, l2_evict_first());
  }
}

// ---------------------------------------------------------------------------
// Warp top-k helpers: (score desc, index asc) ordering.
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool better(double a, int ia, double b, int ib) {
  return a > b || (a == b && ia < ib);
}

// Selects up to `k` best candidates among cand[0..n) (indices 0..n-1 into
// `score`), writing them in order to out[0..k).  `taken` is scratch smem of n
// bytes.  Warp-collective; lane 0 writes.
__device__ void warp_topk(const double *score, int n, int k, unsigned char *taken, int32_t *out,
                          int lane) {
  for (int j = lane; j < n; j += 32) taken[j] = 0;
  __syncwarp();
  for (int t = 0; t < k; ++t) {
    double best = -INFINITY;
    int bi = 0x7fffffff;
    for (int j = lane; j < n; j += 32) {
      if (!taken[j] && better(score[j], j, best, bi)) {
        best = score[j];
        bi = j;
      }
    }
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) {
      double ob = __shfl_xor_sync(0xffffffffu, best, s);
      int oi = __shfl_xor_sync(0xffffffffu, bi, s);
      if (better(ob, oi, best, bi)) {
        best = ob;
        bi = oi;
      }
    }
    if (lane == 0) {
      out[t] = bi;
      taken[bi] = 1;
    }
    __syncwarp();
  }
}

// 16-byte asynchronous copy global -> shared (no registers, many in flight).
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(castdev::smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Sorts the n keys (sk[i], si[i]) of the CTA in place into `better` order
// (score descending, index ascending), a bitonic network over P = the next
// power of two (the tail padded with -inf).  The order is total, so the first
// k entries are exactly the ones warp_topk picks, in the same order.
__device__ void cta_sort_better(double *sk, int32_t *si, int n, int P) {
  for (int i = n + threadIdx.x; i < P; i += blockDim.x) {
    sk[i] = -INFINITY;
    si[i] = 0x7fffffff;
  }
  __syncthreads();
  for (int kk = 2; kk <= P; kk <<= 1)
    for (int j = kk >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < P; i += blockDim.x) {
        const int l = i ^ j;
        if (l > i) {
          const bool i_first = (i & kk) == 0;
          const bool l_better = better(sk[l], si[l], sk[i], si[i]);
          if (i_first == l_better) {  // out of order: swap
            const double td = sk[i];
            sk[i] = sk[l];
            sk[l] = td;
            const int32_t ti = si[i];
            si[i] = si[l];
            si[l] = ti;
          }
        }
      }
      __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// Kernel 2: budget + block-causal selection and the int8/bf16 QK^T policy.
// grid = (nqb, B*H), 128 threads.  Dynamic smem: nkb doubles + nkb bytes.
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(256)
    budget_select_kernel(const double *__restrict__ pooled, const float *__restrict__ block_rms,
                         const float *__restrict__ q_scales, const float *__restrict__ k_scales,
                         int nqb, int nkb, int budget, int maxdeg, int32_t *sel_idx,
                         int32_t *sel_cnt, uint8_t *qk_mode, int policy, float tol, bool stage_k,
                         uint8_t *need_flags) {
  extern __shared__ __align__(16) unsigned char dsm[];
  const int nhist = nkb - nqb;
  int P = 1;
  while (P < nhist) P <<= 1;
  // dynamic shared memory: the history's pooled vectors when they fit
  // (stage_k), the sort keys, then RMS and scales of the key blocks
  double *kst = reinterpret_cast<double *>(dsm);                     // [nhist][D] or none
  double *score = kst + (stage_k ? (size_t)nhist * D : 0);           // [P]
  int32_t *sidx = reinterpret_cast<int32_t *>(score + P);            // [P]
  float *k_rms = reinterpret_cast<float *>(sidx + P);                // [nkb]
  float *k_sc = k_rms + nkb;                                         // [nkb]
  __shared__ double qn[D];
  __shared__ int32_t picks[256];
  const int qb = blockIdx.x, bh = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n_warps = blockDim.x >> 5;
  const double *prow = pooled + (size_t)bh * (nqb + nkb) * D;
  if (stage_k) {  // the history's pooled vectors, all copies in flight at once
    const double *src = prow + (size_t)nqb * D;
    for (int e = threadIdx.x * 2; e < nhist * D; e += blockDim.x * 2) cp_async16(kst + e, src + e);
  }
  for (int d = threadIdx.x; d < D; d += blockDim.x) qn[d] = prow[(size_t)qb * D + d];
  // per key block RMS and scale for the precision policy, fetched up front
  if (qk_mode && policy == CAST_POLICY_AUTO)
    for (int kb = threadIdx.x; kb < nkb; kb += blockDim.x) {
      k_rms[kb] = block_rms[(size_t)bh * (nqb + nkb) + nqb + kb];
      k_sc[kb] = k_scales[(size_t)bh * nkb + kb];
    }
  if (stage_k) cp_async_wait_all();
  __syncthreads();
  for (int kb = warp; kb < nhist; kb += n_warps) {
    const double *b = stage_k ? kst + (size_t)kb * D : prow + (size_t)(nqb + kb) * D;
    double s = warp_dot<D>(qn, b, lane);
    if (lane == 0) {
      score[kb] = s;
      sidx[kb] = kb;
    }
  }
  __syncthreads();
  const int keep = min(budget, nhist);
  cta_sort_better(score, sidx, nhist, P);
  for (int j = threadIdx.x; j < keep; j += blockDim.x) picks[j] = sidx[j];
  __syncthreads();
  int32_t *out = sel_idx + ((size_t)bh * nqb + qb) * maxdeg;
  for (int j = threadIdx.x; j < maxdeg; j += blockDim.x) {
    int val = -1;
    if (j < keep) val = picks[j];
    else if (j < keep + qb + 1) val = nhist + (j - keep);
    out[j] = val;
  }
  if (threadIdx.x == 0) sel_cnt[(size_t)bh * nqb + qb] = keep + qb + 1;
  if (qk_mode && warp == 0) {
    uint8_t mode = policy == CAST_POLICY_INT8 ? 1 : 0;
    if (policy == CAST_POLICY_AUTO) {
      // Predicted logit error of the int8 product (uniform quantisation
      // noise, variance s^2/12 per element) times the logit spread; int8
      // only where every selected block stays below the tolerance.  One lane
      // per selected block, then the warp maximum.
      const float rq = block_rms[(size_t)bh * (nqb + nkb) + qb];
      const float sq = q_scales[(size_t)bh * nqb + qb];
      float worst = 0.0f;
      for (int j = lane; j < keep + qb + 1; j += 32) {
        const int kb = j < keep ? picks[j] : nhist + (j - keep);
        const float rk = k_rms[kb], sk = k_sc[kb];
        const float err = sqrtf((sq * sq * rk * rk + sk * sk * rq * rq) * (1.0f / 12.0f));
        worst = fmaxf(worst, err * rq * rk);
      }
#pragma unroll
      for (int s = 16; s >= 1; s >>= 1) worst = fmaxf(worst, __shfl_xor_sync(0xffffffffu, worst, s));
      mode = worst <= tol ? 1 : 0;
    }
    if (lane == 0) qk_mode[(size_t)bh * nqb + qb] = mode;
    if (need_flags && mode) {  // this query block and every K block it reads need codes
      uint8_t *nf = need_flags + (size_t)bh * (nqb + nkb);
      if (lane == 0) nf[qb] = 1;
      for (int j = lane; j < keep + qb + 1; j += 32) nf[nqb + (j < keep ? picks[j] : nhist + (j - keep))] = 1;
    }
  }
}

// ---------------------------------------------------------------------------
// Compact-path selection (proposed/matrix_curvature_phase_frame_weave.py:
// 5687-5831): every compact block ranks every block by its pooled cosine plus
// 1e6 on the Manhattan-<=1 stencil of the (cell, nh, nw) grid (added to the
// float32 score, as the reference adds it), keeps the first maxdeg in
// (rank descending, index ascending) order, and counts row_degrees[i] of
// them; then the int8/bf16 QK^T policy over those counted blocks.
// grid = (nb, B*H), 256 threads.  Pooled layout [BH][2*nb][D] (queries then
// keys), as pool_quant_kernel writes it with nqb = nkb = nb.
// Dynamic smem: the key blocks' pooled vectors (when stage_k), the sort keys
// [P] and indices [P], the key blocks' RMS and scales [nb] each.
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(256)
    compact_select_kernel(const double *__restrict__ pooled, const float *__restrict__ block_rms,
                          const float *__restrict__ q_scales, const float *__restrict__ k_scales,
                          int nb, int nh, int nw, const int32_t *__restrict__ row_degrees,
                          int maxdeg, int32_t *sel_idx, int32_t *sel_cnt, uint8_t *qk_mode,
                          int policy, float tol, bool stage_k, uint8_t *need_flags) {
  extern __shared__ __align__(16) unsigned char dsm[];
  int P = 1;
  while (P < nb) P <<= 1;
  double *kst = reinterpret_cast<double *>(dsm);                   // [nb][D] or none
  double *score = kst + (stage_k ? (size_t)nb * D : 0);            // [P]
  int32_t *sidx = reinterpret_cast<int32_t *>(score + P);          // [P]
  float *k_rms = reinterpret_cast<float *>(sidx + P);              // [nb]
  float *k_sc = k_rms + nb;                                        // [nb]
  __shared__ double qn[D];
  const int qi = blockIdx.x, bh = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, n_warps = blockDim.x >> 5;
  const double *prow = pooled + (size_t)bh * 2 * nb * D;
  if (stage_k) {
    const double *src = prow + (size_t)nb * D;
    for (int e = threadIdx.x * 2; e < nb * D; e += blockDim.x * 2) cp_async16(kst + e, src + e);
  }
  for (int d = threadIdx.x; d < D; d += blockDim.x) qn[d] = prow[(size_t)qi * D + d];
  const bool auto_policy = qk_mode && policy == CAST_POLICY_AUTO;
  if (auto_policy)
    for (int kb = threadIdx.x; kb < nb; kb += blockDim.x) {
      k_rms[kb] = block_rms[(size_t)bh * 2 * nb + nb + kb];
      k_sc[kb] = k_scales[(size_t)bh * nb + kb];
    }
  if (stage_k) cp_async_wait_all();
  __syncthreads();
  const int spatial = nh * nw;
  const int ti = qi / spatial, hi = (qi % spatial) / nw, wi = qi % nw;
  for (int kb = warp; kb < nb; kb += n_warps) {
    const double *b = stage_k ? kst + (size_t)kb * D : prow + (size_t)(nb + kb) * D;
    const double s = warp_dot<D>(qn, b, lane);
    if (lane == 0) {
      const int tj = kb / spatial, hj = (kb % spatial) / nw, wj = kb % nw;
      const bool local = abs(ti - tj) + abs(hi - hj) + abs(wi - wj) <= 1;
      const float s32 = (float)s;
      score[kb] = (double)(local ? __fadd_rn(s32, 1.0e6f) : s32);
      sidx[kb] = kb;
    }
  }
  __syncthreads();
  cta_sort_better(score, sidx, nb, P);
  const int cnt = min(max(row_degrees[qi], 0), maxdeg);
  int32_t *out = sel_idx + ((size_t)bh * nb + qi) * maxdeg;
  for (int j = threadIdx.x; j < maxdeg; j += blockDim.x) out[j] = j < nb ? sidx[j] : -1;
  if (threadIdx.x == 0) sel_cnt[(size_t)bh * nb + qi] = cnt;
  if (qk_mode && warp == 0) {
    uint8_t mode = policy == CAST_POLICY_INT8 ? 1 : 0;
    if (auto_policy) {
      // the same predicted logit error as the budget rule's policy, over the
      // counted blocks of this row
      const float rq = block_rms[(size_t)bh * 2 * nb + qi];
      const float sq = q_scales[(size_t)bh * nb + qi];
      float worst = 0.0f;
      for (int j = lane; j < cnt; j += 32) {
        const int kb = sidx[j];
        const float rk = k_rms[kb], sk = k_sc[kb];
        const float err = sqrtf((sq * sq * rk * rk + sk * sk * rq * rq) * (1.0f / 12.0f));
        worst = fmaxf(worst, err * rq * rk);
      }
#pragma unroll
      for (int s2 = 16; s2 >= 1; s2 >>= 1) worst = fmaxf(worst, __shfl_xor_sync(0xffffffffu, worst, s2));
      mode = worst <= tol ? 1 : 0;
    }
    if (lane == 0) qk_mode[(size_t)bh * nb + qi] = mode;
    if (need_flags && mode) {
      uint8_t *nf = need_flags + (size_t)bh * 2 * nb;
      if (lane == 0) nf[qi] = 1;
      for (int j = lane; j < cnt; j += 32) nf[nb + sidx[j]] = 1;
    }
  }
}

// ---------------------------------------------------------------------------
// TABA: pooled means over (tt,th,tw) tiles of the visual grid (zero padding
// counts in the mean, as _tile_visual_tensor does), then ranking.
// grid = (nblocks, B*H).
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(kSumLanes *(D / 8), 4)
    pool_grid_kernel(const __nv_bfloat16 *__restrict__ q, const __nv_bfloat16 *__restrict__ k,
                     int T, int Hl, int Wl, int tt, int th, int tw, int nh, int nw, int nblocks,
                     double *pooled /*[BH, 2, nblocks, D]*/) {
  constexpr int kGroups = D / 8;
  __shared__ float red[kSumLanes][D];
  __shared__ double mean_s[D];
  __shared__ double s_denom;
  const int tid = threadIdx.x, grp = tid % kGroups, slot = tid / kGroups;
  const int bh = blockIdx.y;
  const int which = blockIdx.x / nblocks;
  const int blk = blockIdx.x % nblocks;
  const __nv_bfloat16 *X = which == 0 ? q : k;
  const int L = T * Hl * Wl;
  const int bt = blk / (nh * nw), bhh = (blk / nw) % nh, bw = blk % nw;
  const int S = tt * th * tw;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
  for (int r = slot; r < S; r += kSumLanes) {
    const int it = r / (th * tw), ih = (r / tw) % th, iw = r % tw;
    const int t = bt * tt + it, h = bhh * th + ih, w = bw * tw + iw;
    if (t < T && h < Hl && w < Wl) {
      float f[8];
      bf16x8_to_f32(ldg_nc_v4(X + ((size_t)bh * L + ((size_t)t * Hl + h) * Wl + w) * D + grp * 8), f);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], f[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) red[slot][grp * 8 + i] = acc[i];
  __syncthreads();
  if (tid < D) {
    double t = (double)red[0][tid];
#pragma unroll
    for (int p = 1; p < kSumLanes; ++p) t = __dadd_rn(t, (double)red[p][tid]);
    mean_s[tid] = __ddiv_rn(t, (double)S);
  }
  __syncthreads();
  if (tid < 32) {
    double part = __dmul_rn(mean_s[tid], mean_s[tid]);
#pragma unroll
    for (int d = tid + 32; d < D; d += 32) part = __dadd_rn(part, __dmul_rn(mean_s[d], mean_s[d]));
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) part = __dadd_rn(part, __shfl_xor_sync(0xffffffffu, part, s));
    if (tid == 0) s_denom = fmax(__dsqrt_rn(part), kNormEps);
  }
  __syncthreads();
  if (tid < D)
    pooled[(((size_t)bh * 2 + which) * nblocks + blk) * D + tid] = __ddiv_rn(mean_s[tid], s_denom);
}

// grid = (nblocks, B*H), 128 threads; dynamic smem: 2*nblocks doubles + nblocks bytes.
template <int D>
__global__ void __launch_bounds__(128)
    taba_select_kernel(const double *__restrict__ pooled, int nblocks, int nh, int nw,
                       const int32_t *__restrict__ row_degrees, int maxdeg, int32_t *sel_idx,
                       int32_t *sel_cnt, double *scores_out) {
  extern __shared__ __align__(16) unsigned char dsm[];
  double *score = reinterpret_cast<double *>(dsm);
  double *rank = score + nblocks;
  unsigned char *taken = reinterpret_cast<unsigned char *>(rank + nblocks);
  __shared__ double qn[D];
  const int i = blockIdx.x, bh = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const double *qrow = pooled + ((size_t)bh * 2 + 0) * nblocks * D;
  const double *krow = pooled + ((size_t)bh * 2 + 1) * nblocks * D;
  for (int d = threadIdx.x; d < D; d += blockDim.x) qn[d] = qrow[(size_t)i * D + d];
  __syncthreads();
  const int spatial = nh * nw;
  const int ti = i / spatial, hi = (i / nw) % nh, wi = i % nw;
  for (int j = warp; j < nblocks; j += 4) {
    double s = warp_dot<D>(qn, krow + (size_t)j * D, lane);
    if (lane == 0) {
      score[j] = s;
      const int tj = j / spatial, hj = (j / nw) % nh, wj = j % nw;
      const bool local = abs(ti - tj) + abs(hi - hj) + abs(wi - wj) <= 1;
      // The reference adds the stencil bonus to a float32 score.
      const float s32 = (float)s;
      rank[j] = (double)(local ? __fadd_rn(s32, 1.0e6f) : s32);
    }
  }
  __syncthreads();
  if (scores_out)
    for (int j = threadIdx.x; j < nblocks; j += blockDim.x)
      scores_out[((size_t)bh * nblocks + i) * nblocks + j] = score[j];
  if (warp == 0) warp_topk(rank, nblocks, maxdeg, taken, sel_idx + ((size_t)bh * nblocks + i) * maxdeg, lane);
  if (threadIdx.x == 0) sel_cnt[(size_t)bh * nblocks + i] = row_degrees[i];
}

}  // namespace castk
