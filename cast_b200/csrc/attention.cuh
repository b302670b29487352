// Block-sparse flash attention for sm_100a: tcgen05 MMAs with TMEM
// accumulators, TMA-staged tiles (no multicast), online softmax.
//
// One CTA computes up to two 128-row query tiles of one (b*h, query block)
// against the concatenated KV blocks listed for that query block.  Work per
// KV tile j (128 keys):
//   S_i = Q_i K_j^T      int8 x int8 -> s32 (kind::i8) or bf16 -> f32 (kind::f16)
//   P_i = exp2(S_i * c - m_i)  (softmax warpgroup i, written back to TMEM as
//                               bf16 over the S_i columns it was read from)
//   O_i += P_i V_j       bf16 (kind::f16, A = P from TMEM, B = V from SMEM)
//
// Warp roles (384 threads = 3 warpgroups):
//   warps 0-3   softmax + epilogue of query tile 0 (TMEM lanes 0..127)
//   warps 4-7   softmax + epilogue of query tile 1
//   warp 8      TMA producer of Q (once) and the K ring
//   warp 9      MMA issuer (one elected thread) + TMEM allocation
//   warp 10     TMA producer of the V ring (independent of K, so a full V
//               ring never delays the next K tile)
//   warp 11     idle
// The producer/MMA warpgroup gives registers to the two softmax warpgroups
// (setmaxnreg), so a softmax thread holds a whole 128-column S row.
//
// TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512);
// P_i is stored in the lower 64 columns of S_i (128 bf16 keys packed in
// pairs) after the whole S_i row has been read.  MMAs issued by one thread
// execute in issue order, so S_i(j+1) may overwrite P_i(j) once O_i +=
// P_i(j) V_j has been issued before it; and the commit that signals S_i(j+1)
// also covers O_i += P_i(j) V_j, so the softmax can rescale O_i right after
// it sees S_i(j+1).
//
// Lazy rescale: the running max only moves when a tile's max exceeds it by
// more than kRescaleLog2 (in log2 units); probabilities are then bounded by
// 2^kRescaleLog2 and the final normalisation uses the same stale max in
// numerator and denominator, so the result is exact.
#pragma once

#include <climits>

#include "common.cuh"

namespace castk {

constexpr int kAttnThreads = 384;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kVProducerWarp = 10;
constexpr int kSoftmaxRegs = 216;  // setmaxnreg.inc for warpgroups 0-1
constexpr int kServiceRegs = 56;   // setmaxnreg.dec for warpgroup 2
// The CTA's register pool must cover the split: 256*216 + 128*56 = 62464.
constexpr int kRegPoolNeeded = 256 * kSoftmaxRegs + 128 * kServiceRegs;
constexpr int kMaxKStages = 4;
constexpr int kVStages = 3;
constexpr int kMaxBlockList = 256;
constexpr float kRescaleLog2 = 8.0f;

// Shared memory (offsets from the 1024-byte aligned base).  The Q and K
// areas depend on the QK^T precision of the CTA:
//   int8: Q 2 x 16 KB, K ring 4 x 16 KB            (V at 96 KB)
//   bf16: Q 2 x 32 KB, K ring 2 x 32 KB            (V at 128 KB)
// V ring: 3 x 32 KB (bf16 128 keys x 128 dims, two 64-dim swizzled halves).
struct AttnSmem {
  static constexpr int bars = 229376;  // 224 KB: past the largest layout
  // barriers: q_full, k_full[4], k_empty[4], v_full[3], v_empty[3],
  //           s_full[2], p_full[2], o_final
  static constexpr int n_bars = 1 + 2 * kMaxKStages + 2 * kVStages + 2 + 2 + 1;
  static constexpr int tmem_slot = bars + 8 * n_bars;
  static constexpr int blist = (tmem_slot + 16 + 15) / 16 * 16;
  static constexpr int total = blist + 4 * kMaxBlockList;
  static constexpr int alloc = total + 1024;  // alignment slack
};

struct AttnParams {
  const int32_t *indices;
  const int32_t *counts;
  const float *q_scales;
  const float *k_scales;
  const uint8_t *qk_mode;
  const uint8_t *key_valid;
  __nv_bfloat16 *out;
  float *lse;
  int max_degree;
  int BH, Lq, Lk, q_block, k_block, nqb, nkb;
  int q_tiles, k_tiles;  // 128-row tiles per query block / per key block
  int full_pairs;        // q_tiles / 2
  int n_full_items;      // BH * nqb * full_pairs
  int default_mode;      // used when qk_mode == nullptr
  float sm_scale_log2;
};

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// bf16 pair with round-to-nearest (ties up) on the integer pipe: add half an
// ulp of bf16 to the bits of the (non-negative) floats and keep the upper
// halves; `lo` lands in the low 16 bits.
__device__ __forceinline__ uint32_t pack_bf16x2_alu(float lo, float hi) {
  return __byte_perm(__float_as_uint(lo) + 0x8000u, __float_as_uint(hi) + 0x8000u, 0x7632);
}

__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftmaxRegs));
}
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kServiceRegs));
}

// Row max of a full 128-column S row held in registers, times c2 (log2
// units); -inf if every key is masked.  Raw scores are s32 (int8 QK^T) or
// f32 bits (bf16 QK^T).  Eight independent accumulators keep the dependency
// chains short.
template <bool kInt8, bool kMasked>
__device__ __forceinline__ float row_max(const uint32_t (&v)[128], const uint32_t (&kmask)[4],
                                         float c2) {
  if (kInt8) {
    int acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = INT_MIN;
#pragma unroll
    for (int c = 0; c < 128; ++c) {
      int x = (int)v[c];
      if (kMasked) x = ((kmask[c / 32] >> (c % 32)) & 1u) ? x : INT_MIN;
      acc[c & 7] = max(acc[c & 7], x);
    }
#pragma unroll
    for (int s = 4; s >= 1; s >>= 1)
#pragma unroll
      for (int i = 0; i < s; ++i) acc[i] = max(acc[i], acc[i + s]);
    if (acc[0] == INT_MIN) return -INFINITY;
    return (__uint_as_float((uint32_t)acc[0] + 0x4B400000u) - 12582912.0f) * c2;
  } else {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = -INFINITY;
#pragma unroll
    for (int c = 0; c < 128; ++c) {
      float x = __uint_as_float(v[c]);
      if (kMasked) x = ((kmask[c / 32] >> (c % 32)) & 1u) ? x : -INFINITY;
      acc[c & 7] = fmaxf(acc[c & 7], x);
    }
#pragma unroll
    for (int s = 4; s >= 1; s >>= 1)
#pragma unroll
      for (int i = 0; i < s; ++i) acc[i] = fmaxf(acc[i], acc[i + s]);
    return acc[0] * c2;
  }
}

// Probabilities exp2(S*c2 - base) of the row (masked keys 0), packed bf16
// pairs written in place into v[0..63].  Returns the row sum.  For s32 scores
// the int->float conversion is folded into the FFMA:
// float(S) = as_float(S + 0x4B400000) - 1.5*2^23, exact for |S| < 2^22.
template <bool kInt8, bool kMasked>
__device__ __forceinline__ float row_probs(uint32_t (&v)[128], const uint32_t (&kmask)[4],
                                           float c2, float base) {
  const float bias = kInt8 ? fmaf(12582912.0f, c2, base) : base;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int c = 0; c < 64; ++c) {
    const uint32_t a = kInt8 ? v[2 * c] + 0x4B400000u : v[2 * c];
    const uint32_t b = kInt8 ? v[2 * c + 1] + 0x4B400000u : v[2 * c + 1];
    float e0 = fast_exp2(fmaf(__uint_as_float(a), c2, -bias));
    float e1 = fast_exp2(fmaf(__uint_as_float(b), c2, -bias));
    if (kMasked) {
      const uint32_t w = kmask[(2 * c) / 32];
      e0 = ((w >> ((2 * c) % 32)) & 1u) ? e0 : 0.0f;
      e1 = ((w >> ((2 * c + 1) % 32)) & 1u) ? e1 : 0.0f;
    }
    acc[c & 3] += e0 + e1;
    v[c] = pack_bf16x2_alu(e0, e1);
  }
  return (acc[0] + acc[1]) + (acc[2] + acc[3]);
}

__global__ void __launch_bounds__(kAttnThreads, 1)
    rcsa_attention_kernel(const __grid_constant__ CUtensorMap tm_q8,
                          const __grid_constant__ CUtensorMap tm_k8,
                          const __grid_constant__ CUtensorMap tm_q16,
                          const __grid_constant__ CUtensorMap tm_k16,
                          const __grid_constant__ CUtensorMap tm_v, const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bar = reinterpret_cast<uint64_t *>(smem + AttnSmem::bars);
  uint64_t *q_full = bar;
  uint64_t *k_full = bar + 1;
  uint64_t *k_empty = k_full + kMaxKStages;
  uint64_t *v_full = k_empty + kMaxKStages;
  uint64_t *v_empty = v_full + kVStages;
  uint64_t *s_full = v_empty + kVStages;
  uint64_t *p_full = s_full + 2;
  uint64_t *o_final = p_full + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + AttnSmem::tmem_slot);
  int32_t *blist = reinterpret_cast<int32_t *>(smem + AttnSmem::blist);
  int *err = &g_cast_device_error;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // ---- work item (full query-tile pairs first, heaviest query blocks first)
  int bh, qb, pair;
  {
    int x = blockIdx.x;
    if (x < p.n_full_items) {
      pair = x % p.full_pairs;
      const int rest = x / p.full_pairs;
      bh = rest % p.BH;
      qb = p.nqb - 1 - rest / p.BH;
    } else {
      x -= p.n_full_items;
      pair = p.full_pairs;
      bh = x % p.BH;
      qb = p.nqb - 1 - x / p.BH;
    }
  }
  const int t0 = 2 * pair;
  const int nq = min(2, p.q_tiles - t0);
  const int row_item = bh * p.nqb + qb;
  const int n_blocks = min(max(p.counts[row_item], 0), min(p.max_degree, kMaxBlockList));
  const int n_kv = n_blocks * p.k_tiles;
  const int mode = p.qk_mode ? (int)p.qk_mode[row_item] : p.default_mode;  // 1 = int8

  // mode-dependent layout
  const int q_bytes = mode ? 16384 : 32768;  // one 128-row Q tile
  const int k_bytes = mode ? 16384 : 32768;  // one K stage
  const int KS = mode ? 4 : 2;               // K ring depth
  const int q_off = 0;
  const int k_off = 2 * q_bytes;
  const int v_off = k_off + KS * k_bytes;

  if (threadIdx.x == 0) {
    for (int i = 0; i < AttnSmem::n_bars; ++i) castdev::mbar_init(&bar[i], 1);
    castdev::mbar_init(&p_full[0], 4);
    castdev::mbar_init(&p_full[1], 4);
    castdev::fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    castdev::tmem_alloc(tmem_slot, 512);
    castdev::tmem_relinquish();
  }
  for (int j = threadIdx.x; j < n_blocks; j += blockDim.x)
    blist[j] = p.indices[(size_t)row_item * p.max_degree + j];
  if (warp == kProducerWarp && lane == 0) {
    castdev::tma_prefetch_desc(mode ? &tm_q8 : &tm_q16);
    castdev::tma_prefetch_desc(mode ? &tm_k8 : &tm_k16);
    castdev::tma_prefetch_desc(&tm_v);
  }
  __syncthreads();
  castdev::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= 8) {
    setmaxnreg_dec();
    if (warp == kProducerWarp) {
      // ---------------------------------------------------- Q + K producer
      if (lane == 0 && n_kv > 0) {
        bool ok = true;
        const int qrow0 = qb * p.q_block + t0 * 128;
        castdev::mbar_arrive_expect_tx(q_full, nq * q_bytes);
        for (int i = 0; i < nq; ++i) {
          uint8_t *qd = smem + q_off + i * q_bytes;
          if (mode) {
            castdev::tma_load_3d(qd, &tm_q8, q_full, 0, qrow0 + i * 128, bh);
          } else {
            castdev::tma_load_3d(qd, &tm_q16, q_full, 0, qrow0 + i * 128, bh);
            castdev::tma_load_3d(qd + 16384, &tm_q16, q_full, 64, qrow0 + i * 128, bh);
          }
        }
        for (int j = 0; j < n_kv && ok; ++j) {
          const int blk = blist[j / p.k_tiles];
          const int tin = j % p.k_tiles;
          const int krow = (blk >= 0 && blk < p.nkb) ? blk * p.k_block + tin * 128 : 0;
          const int ks = j % KS;
          if (j >= KS) ok = castdev::mbar_wait(&k_empty[ks], ((j / KS) - 1) & 1, err);
          if (!ok) break;
          uint8_t *kd = smem + k_off + ks * k_bytes;
          castdev::mbar_arrive_expect_tx(&k_full[ks], k_bytes);
          if (mode) {
            castdev::tma_load_3d(kd, &tm_k8, &k_full[ks], 0, krow, bh);
          } else {
            castdev::tma_load_3d(kd, &tm_k16, &k_full[ks], 0, krow, bh);
            castdev::tma_load_3d(kd + 16384, &tm_k16, &k_full[ks], 64, krow, bh);
          }
        }
        // Drain: every issued load completes before the CTA may exit.
        castdev::mbar_wait(q_full, 0, err);
        for (int j = max(0, n_kv - KS); j < n_kv; ++j)
          castdev::mbar_wait(&k_full[j % KS], (j / KS) & 1, err);
      }
    } else if (warp == kVProducerWarp) {
      // ---------------------------------------------------- V producer
      if (lane == 0 && n_kv > 0) {
        bool ok = true;
        for (int j = 0; j < n_kv && ok; ++j) {
          const int blk = blist[j / p.k_tiles];
          const int tin = j % p.k_tiles;
          const int krow = (blk >= 0 && blk < p.nkb) ? blk * p.k_block + tin * 128 : 0;
          const int vs = j % kVStages;
          if (j >= kVStages) ok = castdev::mbar_wait(&v_empty[vs], ((j / kVStages) - 1) & 1, err);
          if (!ok) break;
          uint8_t *vd = smem + v_off + vs * 32768;
          castdev::mbar_arrive_expect_tx(&v_full[vs], 32768);
          castdev::tma_load_3d(vd, &tm_v, &v_full[vs], 0, krow, bh);
          castdev::tma_load_3d(vd + 16384, &tm_v, &v_full[vs], 64, krow, bh);
        }
        for (int j = max(0, n_kv - kVStages); j < n_kv; ++j)
          castdev::mbar_wait(&v_full[j % kVStages], (j / kVStages) & 1, err);
      }
    } else if (warp == kMmaWarp) {
      // ---------------------------------------------------- MMA issuer
      if (lane == 0 && n_kv > 0) {
        const uint32_t idesc_s = mode ? castdev::make_idesc(2, 1, 1, 0, 0, 128, 128)
                                      : castdev::make_idesc(1, 1, 1, 0, 0, 128, 128);
        const uint32_t idesc_pv = castdev::make_idesc(1, 1, 1, 0, 1, 128, 128);
        const uint32_t sbase = castdev::smem_u32(smem);
        bool ok = castdev::mbar_wait(q_full, 0, err);
        auto issue_s = [&](int i, int ks) {
          const uint32_t d = tmem + i * 128;
          const uint32_t qa = sbase + q_off + i * q_bytes;
          const uint32_t ka = sbase + k_off + ks * k_bytes;
          if (mode) {
#pragma unroll
            for (int s = 0; s < 4; ++s)
              castdev::mma_i8_ss(d, castdev::smem_desc_sw128(qa + 32 * s, 16, 1024),
                                 castdev::smem_desc_sw128(ka + 32 * s, 16, 1024), idesc_s, s > 0);
          } else {
#pragma unroll
            for (int s = 0; s < 8; ++s) {
              const uint32_t off = (s >> 2) * 16384 + (s & 3) * 32;
              castdev::mma_f16_ss(d, castdev::smem_desc_sw128(qa + off, 16, 1024),
                                  castdev::smem_desc_sw128(ka + off, 16, 1024), idesc_s, s > 0);
            }
          }
        };
        auto issue_pv = [&](int i, int vs, bool first) {
          const uint32_t d = tmem + 256 + i * 128;
          const uint32_t pa = tmem + i * 128;
          const uint32_t va = sbase + v_off + vs * 32768;
#pragma unroll
          for (int s = 0; s < 8; ++s)
            castdev::mma_f16_ts(d, pa + 8 * s, castdev::smem_desc_sw128(va + 2048 * s, 16384, 1024),
                                idesc_pv, (!first || s > 0) ? 1u : 0u);
        };
        if (ok) ok = castdev::mbar_wait(&k_full[0], 0, err);
        if (ok) {
          castdev::tc_fence_after();
          for (int i = 0; i < nq; ++i) {
            issue_s(i, 0);
            castdev::tc_commit(&s_full[i]);
          }
          castdev::tc_commit(&k_empty[0]);
        }
        for (int j = 0; j < n_kv && ok; ++j) {
          const int vs = j % kVStages;
          ok = castdev::mbar_wait(&v_full[vs], (j / kVStages) & 1, err);
          for (int i = 0; i < nq && ok; ++i) {
            ok = castdev::mbar_wait(&p_full[i], j & 1, err);
            if (!ok) break;
            castdev::tc_fence_after();
            issue_pv(i, vs, j == 0);
            if (j + 1 < n_kv) {
              const int ks = (j + 1) % KS;
              if (i == 0) {
                ok = castdev::mbar_wait(&k_full[ks], ((j + 1) / KS) & 1, err);
                if (!ok) break;
                castdev::tc_fence_after();
              }
              issue_s(i, ks);
              castdev::tc_commit(&s_full[i]);
            }
          }
          castdev::tc_commit(&v_empty[vs]);
          if (j + 1 < n_kv) castdev::tc_commit(&k_empty[(j + 1) % KS]);
        }
        castdev::tc_commit(o_final);
      }
    }
  } else {
    setmaxnreg_inc();
    // ------------------------------------------------------------ softmax
    const int ti = warp >> 2;  // query tile handled by this warpgroup
    const int row = (warp & 3) * 32 + lane;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + ti * 128;
    const uint32_t o_addr = tmem + lane_off + 256 + ti * 128;
    const bool active = ti < nq;
    const int qrow_in_block = (t0 + ti) * 128 + row;
    const int qrow = qb * p.q_block + qrow_in_block;
    const bool row_valid = active && qrow_in_block < p.q_block && qrow < p.Lq;
    const float qscale = mode ? p.q_scales[row_item] : 1.0f;
    float m_run = -INFINITY, l_run = 0.0f;
    bool ok = true;
    if (active) {
      for (int j = 0; j < n_kv; ++j) {
        const int blk = blist[j / p.k_tiles];
        const int tin = j % p.k_tiles;
        const bool blk_ok = blk >= 0 && blk < p.nkb;
        const int krow = blk_ok ? blk * p.k_block + tin * 128 : 0;
        const int valid_cols = blk_ok ? min(128, min(p.k_block - tin * 128, p.Lk - krow)) : 0;
        const float c2 = (mode && blk_ok ? qscale * p.k_scales[(size_t)bh * p.nkb + blk] : 1.0f) *
                         p.sm_scale_log2;
        // Key mask of this tile: columns >= valid_cols, and key_valid == 0.
        uint32_t kmask[4];
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const int lo = valid_cols - 32 * w;
          kmask[w] = lo >= 32 ? 0xffffffffu : (lo <= 0 ? 0u : ((1u << lo) - 1u));
        }
        if (p.key_valid && valid_cols > 0) {
          const uint4 *kv4 = reinterpret_cast<const uint4 *>(p.key_valid + krow);
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            uint32_t bits = 0;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const uint4 b = kv4[2 * w + h];
              const uint32_t words[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
              for (int q4 = 0; q4 < 4; ++q4)
#pragma unroll
                for (int by = 0; by < 4; ++by)
                  if ((words[q4] >> (8 * by)) & 0xFFu) bits |= 1u << (16 * h + 4 * q4 + by);
            }
            kmask[w] &= bits;
          }
        }
        const bool full_tile = (kmask[0] & kmask[1] & kmask[2] & kmask[3]) == 0xffffffffu;

        ok = __all_sync(0xffffffffu, castdev::mbar_wait(&s_full[ti], j & 1, err));
        if (!ok) break;
        castdev::tc_fence_after();
        uint32_t v[128];
#pragma unroll
        for (int w = 0; w < 4; ++w)
          castdev::tmem_ld32(s_addr + 32 * w, *reinterpret_cast<uint32_t(*)[32]>(&v[32 * w]));
        castdev::tmem_wait_ld();

        const float m_tile = mode ? (full_tile ? row_max<true, false>(v, kmask, c2)
                                               : row_max<true, true>(v, kmask, c2))
                                  : (full_tile ? row_max<false, false>(v, kmask, c2)
                                               : row_max<false, true>(v, kmask, c2));
        const bool need = m_tile > m_run + kRescaleLog2;
        if (__any_sync(0xffffffffu, need)) {
          const float m_new = fmaxf(m_run, m_tile);
          const float alpha = (m_run == -INFINITY) ? (m_new == -INFINITY ? 1.0f : 0.0f)
                                                   : fast_exp2(m_run - m_new);
          if (j > 0) {
#pragma unroll 1
            for (int cc = 0; cc < 4; ++cc) {
              uint32_t o[32];
              castdev::tmem_ld32(o_addr + 32 * cc, o);
              castdev::tmem_wait_ld();
#pragma unroll
              for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
              castdev::tmem_st32(o_addr + 32 * cc, o);
            }
            castdev::tmem_wait_st();
          }
          l_run *= alpha;
          m_run = m_new;
        }
        const float base = (m_run == -INFINITY) ? 0.0f : m_run;
        const float sum = mode ? (full_tile ? row_probs<true, false>(v, kmask, c2, base)
                                            : row_probs<true, true>(v, kmask, c2, base))
                               : (full_tile ? row_probs<false, false>(v, kmask, c2, base)
                                            : row_probs<false, true>(v, kmask, c2, base));
        castdev::tmem_st32(s_addr, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
        castdev::tmem_st32(s_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
        l_run += sum;
        castdev::tmem_wait_st();
        castdev::tc_fence_before();
        __syncwarp();
        if (lane == 0) castdev::mbar_arrive(&p_full[ti]);
      }
    }
    // ------------------------------------------------------------ epilogue
    if (active && ok) {
      if (n_kv > 0) {
        ok = __all_sync(0xffffffffu, castdev::mbar_wait(o_final, 0, err));
        castdev::tc_fence_after();
      }
      const float inv_l = l_run > 0.0f ? 1.0f / l_run : 0.0f;
      __nv_bfloat16 *orow = p.out + ((size_t)bh * p.Lq + qrow) * 128;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t o[32];
        if (n_kv > 0 && ok) {
          castdev::tmem_ld32(o_addr + 32 * cc, o);
          castdev::tmem_wait_ld();
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) o[c] = 0u;
        }
        if (row_valid) {
          uint4 w[4];
          uint32_t *wp = reinterpret_cast<uint32_t *>(w);
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            __nv_bfloat162 h2 = __floats2bfloat162_rn(__uint_as_float(o[2 * c]) * inv_l,
                                                      __uint_as_float(o[2 * c + 1]) * inv_l);
            wp[c] = *reinterpret_cast<uint32_t *>(&h2);
          }
          uint4 *dst = reinterpret_cast<uint4 *>(orow + 32 * cc);
#pragma unroll
          for (int c = 0; c < 4; ++c) dst[c] = w[c];
        }
      }
      if (row_valid && p.lse)
        p.lse[(size_t)bh * p.Lq + qrow] = l_run > 0.0f ? m_run + __log2f(l_run) : -INFINITY;
    }
  }

  __syncthreads();
  if (warp == kMmaWarp) {
    castdev::tc_fence_after();
    castdev::tmem_dealloc(tmem, 512);
  }
}

}  // namespace castk
