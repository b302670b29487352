// Block-sparse flash attention for sm_100a: tcgen05 MMAs with TMEM
// accumulators, TMA-staged tiles (no multicast), online softmax.
//
// One CTA computes up to two 128-row query tiles of one (b*h, query block)
// against the concatenated KV blocks listed for that query block.  TMA moves
// K and V in tiles of 128 keys; the MMAs and the softmax step through them in
// halves of 64 keys (step h = tile h/2, half h%2):
//   S_i(h) = Q_i K_h^T    int8 x int8 -> s32 (kind::i8) or bf16 -> f32 (kind::f16)
//   P_i(h) = exp2(S_i(h) * c - m_i)   (softmax warpgroup i; bf16 pairs written
//                                      back over the first 32 columns of S_i(h))
//   O_i   += P_i(h) V_h   bf16 (kind::f16, A = P from TMEM, B = V from SMEM)
//
// Warp roles (384 threads = 3 warpgroups):
//   warps 0-3   softmax + epilogue of query tile 0 (TMEM lanes 0..127)
//   warps 4-7   softmax + epilogue of query tile 1
//   warp 8      TMA producer of Q (once) and the K ring
//   warp 9      MMA issuer of query tile 0 (one thread) + TMEM allocation
//   warp 10     TMA producer of the V ring
//   warp 11     MMA issuer of query tile 1 (one thread)
// Each query tile has its own issuing thread, so neither tile's MMAs wait
// behind the other tile's barrier polls.
//
// TMEM (512 columns): O0 [0,128) O1 [128,256), then two S buffers of 64
// columns per query tile: S_i buffer b at 256 + 128 i + 64 b.  S_i(h) lives in
// buffer h%2, so the MMA thread issues S_i(h+2) right after O_i += P_i(h) V_h:
// while the softmax works on step h, the tensor core has already produced
// S_i(h+1), and the softmax never waits for its own PV.  MMAs issued by one
// thread execute in issue order, so S_i(h+2) may overwrite P_i(h) once the PV
// that reads it has been issued.
//
// Lazy rescale: the running max only moves when a step's max exceeds it by
// more than kRescaleLog2 (in log2 units); probabilities are then bounded by
// 2^kRescaleLog2 and the final normalisation uses the same stale max in
// numerator and denominator, so the result is exact.  A rescale of O_i first
// waits for the PV of the previous step (pv_done), which is still in flight.
#pragma once

#include <climits>
#include <type_traits>

#include "common.cuh"

namespace castk {

#ifndef CAST_ATTN_HEAD_GROUP
#define CAST_ATTN_HEAD_GROUP (1 << 20)
#endif
constexpr int kAttnThreads = 384;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kVProducerWarp = 10;
constexpr int kMmaWarp1 = 11;  // MMA issuer of query tile 1
constexpr int kMaxKStages = 4;
constexpr int kVStages = 3;
constexpr int kMaxBlockList = 256;
constexpr float kRescaleLog2 = 8.0f;
constexpr int kMaxSplitItems = 512;  // items cut into parts in one launch
constexpr int kMaxItemParts = 64;    // parts of one cut item
// Partial result of one part: O of both query tiles (fp32, [tile][column]
// [row], so a warp's 32 rows are contiguous), then per tile the running max
// and the row sum of its 128 rows.
constexpr int kPartSlotFloats = 2 * 128 * 128 + 2 * 2 * 128;
constexpr int kMaxPeers = 7;  // other ranks a launch writes its outputs to

// Shared memory (offsets from the 1024-byte aligned base).  The Q and K
// areas depend on the QK^T precision of the CTA:
//   int8: Q 2 x 16 KB, K ring 4 x 16 KB            (V at 96 KB)
//   bf16: Q 2 x 32 KB, K ring 2 x 32 KB            (V at 128 KB)
// V ring: 3 x 32 KB (bf16 128 keys x 128 dims, two 64-dim swizzled halves).
struct AttnSmem {
  static constexpr int bars = 229376;  // 224 KB: past the largest layout
  // barriers: q_full, k_full[4], k_empty[4], v_full[3], v_empty[3],
  //           s_full[2][2], p_full[2][2], pv_done[2][2], mma_drain[2], merge
  static constexpr int n_bars = 1 + 2 * kMaxKStages + 2 * kVStages + 4 + 4 + 4 + 2 + 1;
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
  int nkb_full;          // key blocks read through the block-structured value map (0: none)
  int q_tiles, k_tiles;  // 128-row tiles per query block / per key block
  int full_pairs;        // q_tiles / 2
  int n_full_items;      // BH * nqb * full_pairs
  int default_mode;      // used when qk_mode == nullptr
  float sm_scale_log2;
  // Work split.  CTA x < n_whole runs item x over all its key tiles.  Item
  // n_whole + s (s < n_split) is cut along its key tiles into the parts
  // part_first[s] .. part_first[s+1]-1, run by CTAs n_whole + part; part j of
  // n covers key tiles [j*T/n, (j+1)*T/n) of the T = part_tiles[s] the host
  // planned, the last part everything from there on.  Each part leaves its
  // partial result in slot `part` of part_ws; the last part of the item to
  // finish (counted in part_counter[s], zero between launches) merges them.
  int n_whole, n_split;
  // Converted pairs (n_conv > 0, no cut items then): the last n_conv pair
  // items run as single query tiles, after the native single tiles: CTAs
  // [0, n_full_items - n_conv) pairs, then the n_items - n_full_items
  // single tiles, then two CTAs per converted pair (tile 2*pair, 2*pair+1).
  int n_conv, n_items;
  int *part_counter;
  float *part_ws;
  uint16_t part_first[kMaxSplitItems + 1];
  uint16_t part_tiles[kMaxSplitItems];
  // Head-sharded all-gather fused into the epilogue (n_peers > 0): every
  // output row is also stored, over NVLink, at the same offset of each
  // peer's gathered buffer (peer_out[r] is this rank's slot there).  Every
  // CTA fences its stores at system scope and takes a ticket; the launch's
  // last CTA then raises this rank's flag in every peer to this call's
  // number (*calls + 1, a release store) and resets the ticket.  The call
  // counter lives on the device, so a captured graph replays correctly.
  int n_peers;
  const uint32_t *calls;
  uint32_t *done_ticket;
  __nv_bfloat16 *peer_out[kMaxPeers];
  uint32_t *peer_flag[kMaxPeers];
};

// Work items are ordered in groups of kHeadGroup heads: within a group,
// query blocks heaviest first (the last query block selects the most key
// blocks), then head, then tile pair.  A group's CTAs run close together, so
// the key/value blocks its heads selected are read from DRAM once and shared
// through L2, while the order inside a group keeps the heavy items early.
constexpr int kHeadGroup = CAST_ATTN_HEAD_GROUP;

// (bh, query block, pair) of item y (pairs: per = full_pairs; single tiles:
// per = 1) in the grouped order above.
__host__ __device__ __forceinline__ void item_coords(int y, int BH, int nqb, int per, int &bh,
                                                     int &qb, int &pair) {
  const int G = kHeadGroup < BH ? kHeadGroup : BH;
  const int group_items = G * nqb * per;
  const int g = y / group_items;
  const int gh = min(G, BH - g * G);
  const int r = y - g * group_items;
  pair = r % per;
  const int rest = r / per;
  bh = g * G + rest % gh;
  qb = nqb - 1 - rest / gh;
}

// First key tile of part j of n over T planned tiles.
__device__ __forceinline__ int part_lo(int j, int T, int n) {
  return (int)(((long long)j * T) / n);
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h2 = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&h2);
}

// Row max of a 64-column S step held in registers, times c2 (log2 units);
// -inf if every key is masked.  Raw scores are s32 (int8 QK^T) or f32 bits
// (bf16 QK^T).  Eight independent accumulators keep the chains short.
template <bool kInt8, bool kMasked>
__device__ __forceinline__ float row_max(const uint32_t (&v)[64], const uint32_t (&kmask)[2],
                                         float c2) {
  if (kInt8) {
    int acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = INT_MIN;
#pragma unroll
    for (int c = 0; c < 64; ++c) {
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
    for (int c = 0; c < 64; ++c) {
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

// Shared-memory descriptor as (lo, hi) words: hi is fixed by the LBO/SBO
// strides, and lo = start>>4 | LBO>>4 << 16, so an operand `off` bytes further
// on is lo + off/16 (smem addresses stay below 2^18, so nothing carries).
struct DescW {
  uint32_t lo, hi;
  __device__ __forceinline__ uint64_t at(uint32_t off) const {
    return ((uint64_t)hi << 32) | (uint64_t)(lo + (off >> 4));
  }
};
__device__ __forceinline__ DescW desc_words(uint32_t addr, uint32_t lbo) {
  const uint64_t d = castdev::smem_desc_sw128(addr, lbo, 1024);
  return DescW{(uint32_t)d, (uint32_t)(d >> 32)};
}

// Position in the shared K/V ring of an issuer's (or softmax warpgroup's)
// t-th 128-key tile.  Pair items (two query tiles, one key list): both tiles
// read every ring tile, position t.  Split items (one query tile whose key
// tiles are split between the two warpgroups, A = the first n_a, B = the
// last n_b, n_a - n_b in {0, 1}): ring order A0 B0 A1 B1 ... then the rest of
// A, so warpgroup i's t-th tile sits at 2t + i while t < n_b, and A's tail at
// n_b + t.
struct RingMap {
  int split, i, n_a, n_b;
  __device__ __forceinline__ int pos(int t) const {
    return !split ? t : (t < n_b ? 2 * t + i : n_b + t);
  }
  // key tile (index into the item's concatenated key list) at ring position r
  __device__ __forceinline__ int key_tile(int r) const {
    return !split ? r : (r < 2 * n_b ? ((r & 1) ? n_a + (r >> 1) : (r >> 1)) : r - n_b);
  }
};

// The MMA issuer of query tile i (one thread per tile).  Per 64-key step h:
//   wait P_i(h); O_i += P_i(h) V_h; commit pv_done; then S_i(h+2) into the S
//   buffer P_i(h) came from (issued after the PV that reads it); commit
//   s_full.  K and V stages are released by commits after their last use;
//   their "empty" barriers count one arrival per active tile.
// Returns false if a wait gave up.
template <int kInt8>
__device__ __forceinline__ bool mma_issuer(int i, RingMap ring, uint32_t tmem, uint32_t sbase,
                                           int n_steps, int q_bytes, int k_off, int v_off,
                                           uint64_t *q_full,
                                           uint64_t *k_full, uint64_t *k_empty, uint64_t *v_full,
                                           uint64_t *v_empty, uint64_t *s_full, uint64_t *p_full,
                                           uint64_t *pv_done, int *err) {
  constexpr int KS = kInt8 ? 4 : 2;              // K ring depth
  constexpr int kKBytes = kInt8 ? 16384 : 32768;  // one K stage
  constexpr uint32_t idesc_s = kInt8 ? castdev::make_idesc(2, 1, 1, 0, 0, 128, 64)
                                     : castdev::make_idesc(1, 1, 1, 0, 0, 128, 64);
  constexpr uint32_t idesc_pv = castdev::make_idesc(1, 1, 1, 0, 1, 128, 128);
  const DescW qd = desc_words(sbase + (ring.split ? 0 : i * q_bytes), 16);
  const DescW kd = desc_words(sbase + k_off, 16);     // + stage * kKBytes + half * 8192
  const DescW vd = desc_words(sbase + v_off, 16384);  // + stage * 32768 + half * 8192
  const uint32_t o_col = tmem + i * 128;
  const uint32_t s_col = tmem + 256 + i * 128;
  uint64_t *my_s_full = s_full + 2 * i;
  uint64_t *my_p_full = p_full + 2 * i;
  uint64_t *my_pv_done = pv_done + 2 * i;

  // S_i of one half of the key tile at ring position r into S buffer `half`
  auto issue_s = [&](int r, int half) {
    const uint32_t d = s_col + half * 64;
    const uint32_t ko = ((uint32_t)r & (KS - 1)) * kKBytes + half * 8192;
    if (kInt8) {
#pragma unroll
      for (int s = 0; s < 4; ++s)
        castdev::mma_i8_ss(d, qd.at(32 * s), kd.at(ko + 32 * s), idesc_s, s > 0);
    } else {
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const uint32_t off = (s >> 2) * 16384 + (s & 3) * 32;
        castdev::mma_f16_ss(d, qd.at(off), kd.at(ko + off), idesc_s, s > 0);
      }
    }
  };
  const int n_tiles = n_steps / 2;

  int rk = ring.pos(0);  // ring position of the next key tile to multiply
  if (!castdev::mbar_wait(q_full, 0, err) ||
      !castdev::mbar_wait(&k_full[rk & (KS - 1)], (rk / KS) & 1, err))
    return false;
  castdev::tc_fence_after();
  issue_s(rk, 0);
  castdev::tc_commit(&my_s_full[0]);
  issue_s(rk, 1);
  castdev::tc_commit(&my_s_full[1]);
  castdev::tc_commit(&k_empty[rk & (KS - 1)]);

  // Per key tile t: steps 2t and 2t+1 (its two halves).  Ring positions,
  // stages and phases are worked out once per tile.
  for (int t = 0; t < n_tiles; ++t) {
    const int rv = ring.pos(t);  // ring position of this tile's V
    const int vs = rv % kVStages;
    const bool more = t + 1 < n_tiles;
    if (more) rk = ring.pos(t + 1);
    if (!castdev::mbar_wait(&v_full[vs], (rv / kVStages) & 1, err)) return false;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      if (!castdev::mbar_wait(&my_p_full[half], t & 1, err)) return false;
      castdev::tc_fence_after();
      const uint32_t vo = vs * 32768 + half * 8192;
      const uint32_t pa = s_col + half * 64;
#pragma unroll
      for (int s = 0; s < 4; ++s)
        castdev::mma_f16_ts(o_col, pa + 8 * s, vd.at(vo + 2048 * s), idesc_pv, (t | half | s) != 0);
      castdev::tc_commit(&my_pv_done[half]);
      if (more) {
        // S of the next tile's same half, into the buffer this PV read
        if (half == 0) {
          if (!castdev::mbar_wait(&k_full[rk & (KS - 1)], (rk / KS) & 1, err)) return false;
          castdev::tc_fence_after();
        }
        issue_s(rk, half);
        castdev::tc_commit(&my_s_full[half]);
      }
    }
    castdev::tc_commit(&v_empty[vs]);
    if (more) castdev::tc_commit(&k_empty[rk & (KS - 1)]);
  }
  return true;
}

// Packed f32x2 arithmetic (two fp32 lanes per instruction).
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t r, float &lo, float &hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// acc + the low (high) bf16 half of a packed pair, widened exactly to fp32:
// one mixed-precision add (sm_100) instead of an unpack and an add.
__device__ __forceinline__ float add_bf16_lo(uint32_t pk, float acc) {
  float r;
  asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %1;\n\tadd.rn.f32.bf16 %0, lo, %2;\n\t}"
      : "=f"(r) : "r"(pk), "f"(acc));
  return r;
}
__device__ __forceinline__ float add_bf16_hi(uint32_t pk, float acc) {
  float r;
  asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %1;\n\tadd.rn.f32.bf16 %0, hi, %2;\n\t}"
      : "=f"(r) : "r"(pk), "f"(acc));
  return r;
}

// The fast path accepts a step whose probabilities (against a running max
// that may be stale) sum to at most 2^kFastSumLog2: each is then at most
// 2^16, far from overflow in bf16 and in the fp32 sums and accumulators, and
// the final normalisation does not depend on the scale.  A larger sum (or
// inf) sends the warp to the exact path.
constexpr float kFastSumLimit = 65536.0f;

// Probabilities exp2(S*c2 - base) of a 64-key step in one pass: packed FFMA
// for the exponent, MUFU exp2, bf16 pairs written in place into v[0..31],
// packed row sums of those bf16 values.  Returns their sum.  For s32 scores the int->float
// conversion is folded into the FFMA: float(S) = as_float(S + 0x4B400000) -
// 1.5*2^23, exact for |S| < 2^22.
template <bool kInt8, bool kMasked>
__device__ __forceinline__ float step_probs(uint32_t (&v)[64], const uint32_t (&kmask)[2],
                                            float c2, float base) {
  const float bias = kInt8 ? fmaf(12582912.0f, c2, base) : base;
  const uint64_t c2x2 = f2_pack(c2, c2);
  const uint64_t nbx2 = f2_pack(-bias, -bias);
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int c = 0; c < 32; ++c) {
    const uint32_t a = kInt8 ? v[2 * c] + 0x4B400000u : v[2 * c];
    const uint32_t b = kInt8 ? v[2 * c + 1] + 0x4B400000u : v[2 * c + 1];
    float x0, x1;
    f2_unpack(f2_fma(f2_pack(__uint_as_float(a), __uint_as_float(b)), c2x2, nbx2), x0, x1);
    float e0 = fast_exp2(x0);
    float e1 = fast_exp2(x1);
    if (kMasked) {
      const uint32_t w = kmask[(2 * c) / 32];
      e0 = ((w >> ((2 * c) % 32)) & 1u) ? e0 : 0.0f;
      e1 = ((w >> ((2 * c + 1) % 32)) & 1u) ? e1 : 0.0f;
    }
    // the row sum adds the bf16-rounded probabilities the P.V MMA reads, so
    // the normalised weights sum to one: a row dominated by a few keys then
    // reproduces their values instead of carrying the rounding of their
    // weights (up to 2^-9 relative) into the output
    const uint32_t pk = pack_bf16x2(e0, e1);
    acc[2 * (c & 3)] = add_bf16_lo(pk, acc[2 * (c & 3)]);
    acc[2 * (c & 3) + 1] = add_bf16_hi(pk, acc[2 * (c & 3) + 1]);
    v[c] = pk;
  }
  return ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
}

template <bool kInt8>
__device__ __forceinline__ float step_probs_any(uint32_t (&v)[64], const uint32_t (&kmask)[2],
                                                bool full, float c2, float base) {
  return full ? step_probs<kInt8, false>(v, kmask, c2, base)
              : step_probs<kInt8, true>(v, kmask, c2, base);
}

// A CTA's exit with the fused all-gather: its ticket; the launch's last CTA
// raises this rank's flag in every peer.  Every CTA fenced its own stores at
// system scope before taking its ticket.
__device__ __forceinline__ void peer_ticket(const AttnParams &p) {
  const uint32_t t = atomicAdd(p.done_ticket, 1u);
  if (t == gridDim.x - 1) {
    __threadfence_system();
    const uint32_t call = *reinterpret_cast<const volatile uint32_t *>(p.calls) + 1u;
    for (int r = 0; r < p.n_peers; ++r) castdev::st_release_sys(p.peer_flag[r], call);
    atomicExch(p.done_ticket, 0u);
  }
}

__global__ void __launch_bounds__(kAttnThreads, 1)
    rcsa_attention_kernel(const __grid_constant__ CUtensorMap tm_q8,
                          const __grid_constant__ CUtensorMap tm_k8,
                          const __grid_constant__ CUtensorMap tm_q16,
                          const __grid_constant__ CUtensorMap tm_k16,
                          const __grid_constant__ CUtensorMap tm_v,
                          const __grid_constant__ CUtensorMap tm_vb, const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bar = reinterpret_cast<uint64_t *>(smem + AttnSmem::bars);
  uint64_t *q_full = bar;
  uint64_t *k_full = bar + 1;
  uint64_t *k_empty = k_full + kMaxKStages;
  uint64_t *v_full = k_empty + kMaxKStages;
  uint64_t *v_empty = v_full + kVStages;
  uint64_t *s_full = v_empty + kVStages;  // [tile * 2 + buffer]
  uint64_t *p_full = s_full + 4;          // [tile * 2 + buffer]
  uint64_t *pv_done = p_full + 4;         // [tile * 2 + buffer]
  uint64_t *mma_drain = pv_done + 4;
  uint64_t *merge_bar = mma_drain + 2;  // split items: warpgroup 1's partial result is ready
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + AttnSmem::tmem_slot);
  volatile uint32_t *part_flag = tmem_slot + 1;  // this CTA merges its cut item
  int32_t *blist = reinterpret_cast<int32_t *>(smem + AttnSmem::blist);
  // set when one of this CTA's waits gives up, so the others stop too
  int *err = reinterpret_cast<int *>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // ---- work item (full query-tile pairs first, heaviest query blocks first)
  // and, for a cut item, which part of it
  int x = blockIdx.x, split_idx = -1, part = 0, n_parts = 1, planned = 0;
  int conv_tile = -1;  // converted pair: which of its two tiles this CTA runs
  if (p.n_conv > 0) {
    const int kept = p.n_full_items - p.n_conv;
    const int singles = p.n_items - p.n_full_items;
    if (x >= kept + singles) {
      const int j = x - kept - singles;
      x = kept + j / 2;
      conv_tile = j & 1;
    } else if (x >= kept) {
      x = p.n_full_items + (x - kept);
    }
  } else if (x >= p.n_whole) {
    const int b = x - p.n_whole;
    int lo = 0, hi = p.n_split;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if ((int)p.part_first[mid] <= b)
        lo = mid;
      else
        hi = mid;
    }
    split_idx = lo;
    part = b - (int)p.part_first[lo];
    n_parts = (int)p.part_first[lo + 1] - (int)p.part_first[lo];
    planned = p.part_tiles[lo];
    x = p.n_whole + lo;
  }
  int bh, qb, pair;
  {
    if (x < p.n_full_items) {
      item_coords(x, p.BH, p.nqb, p.full_pairs, bh, qb, pair);
    } else {
      int unused;
      item_coords(x - p.n_full_items, p.BH, p.nqb, 1, bh, qb, unused);
      pair = p.full_pairs;
    }
  }
  const int t0 = 2 * pair + max(conv_tile, 0);
  const int nq = conv_tile >= 0 ? 1 : min(2, p.q_tiles - t0);
  const int row_item = bh * p.nqb + qb;
  const int n_blocks = min(max(p.counts[row_item], 0), min(p.max_degree, kMaxBlockList));
  const int n_kv_item = n_blocks * p.k_tiles;  // 128-key tiles of the item
  // This CTA's key tiles [kt_lo, kt_lo + n_kv), and the number of the item's
  // parts that have any (n_live; 1 = this CTA writes the output itself).
  int kt_lo = 0, n_kv = n_kv_item, n_live = 1;
  if (split_idx >= 0) {
    const int lo = part_lo(part, planned, n_parts);
    const int hi = part + 1 == n_parts ? INT_MAX : part_lo(part + 1, planned, n_parts);
    kt_lo = min(lo, n_kv_item);
    n_kv = min(hi, n_kv_item) - kt_lo;
    n_live = 0;
    for (int j = 0; j < n_parts; ++j) n_live += part_lo(j, planned, n_parts) < n_kv_item;
    if ((n_kv_item == 0 && part > 0) || (n_kv_item > 0 && n_kv == 0)) {
      // no key tiles here (part 0 of an empty item writes its zero rows)
      if (p.n_peers > 0 && threadIdx.x == 0) peer_ticket(p);
      return;
    }
    if (n_kv_item == 0) n_live = 1;
  }
  // A single query tile (the last of an odd tile count) splits its key tiles
  // between the two warpgroups (split item), whose partial results are merged
  // at the end; a pair gives each warpgroup its own query tile.
  const bool split = nq == 1 && n_kv >= 2;
  const int n_a = split ? (n_kv + 1) / 2 : n_kv;  // key tiles of warpgroup / issuer 0
  const int n_b = split ? n_kv - n_a : n_kv;      // key tiles of warpgroup / issuer 1
  const int n_groups = split ? 2 : nq;            // active warpgroups and issuers
  const RingMap ring0{split ? 1 : 0, 0, n_a, n_b};
  const int mode = p.qk_mode ? (int)p.qk_mode[row_item] : p.default_mode;  // 1 = int8

  // mode-dependent layout
  const int q_bytes = mode ? 16384 : 32768;  // one 128-row Q tile
  const int k_bytes = mode ? 16384 : 32768;  // one K stage
  const int KS = mode ? 4 : 2;               // K ring depth
  const int q_off = 0;
  const int k_off = 2 * q_bytes;
  const int v_off = k_off + KS * k_bytes;

  if (warp == kProducerWarp && lane == 0) {
    // The producer thread initialises the barriers and starts the Q load
    // before the CTA-wide sync, so the load overlaps the rest of the set-up.
    *err = 0;
    for (int i = 0; i < AttnSmem::n_bars; ++i) castdev::mbar_init(&bar[i], 1);
    for (int i = 0; i < 4; ++i) castdev::mbar_init(&p_full[i], 4);
    castdev::mbar_init(merge_bar, 4);
    // a K or V stage is free once every issuer reading it has done so (both
    // for a pair, the one owning that ring tile for a split item)
    for (int i = 0; i < kMaxKStages; ++i) castdev::mbar_init(&k_empty[i], split ? 1 : nq);
    for (int i = 0; i < kVStages; ++i) castdev::mbar_init(&v_empty[i], split ? 1 : nq);
    castdev::fence_barrier_init();
    castdev::tma_prefetch_desc(mode ? &tm_q8 : &tm_q16);
    castdev::tma_prefetch_desc(mode ? &tm_k8 : &tm_k16);
    castdev::tma_prefetch_desc(&tm_v);
    if (p.nkb_full > 0) castdev::tma_prefetch_desc(&tm_vb);
    if (n_kv > 0) {
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
    }
  }
  if (warp == kMmaWarp) {
    castdev::tmem_alloc(tmem_slot, 512);
    castdev::tmem_relinquish();
  }
  // the whole list row (not only `counts` entries), so these loads need not
  // wait for the count
  for (int j = threadIdx.x; j < min(p.max_degree, kMaxBlockList); j += blockDim.x)
    blist[j] = p.indices[(size_t)row_item * p.max_degree + j];
  __syncthreads();
  castdev::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= 8) {
    if (warp == kProducerWarp) {
      // ---------------------------------------------------- Q + K producer
      if (lane == 0 && n_kv > 0) {  // (Q is already on its way)
        int issued = 0;
        for (int j = 0; j < n_kv; ++j) {  // ring position j
          const int kt = kt_lo + ring0.key_tile(j);
          const int blk = blist[kt / p.k_tiles];
          const int tin = kt % p.k_tiles;
          const int krow = (blk >= 0 && blk < p.nkb) ? blk * p.k_block + tin * 128 : 0;
          const int ks = j % KS;
          if (j >= KS && !castdev::mbar_wait(&k_empty[ks], ((j / KS) - 1) & 1, err)) break;
          uint8_t *kd = smem + k_off + ks * k_bytes;
          castdev::mbar_arrive_expect_tx(&k_full[ks], k_bytes);
          if (mode) {
            castdev::tma_load_3d(kd, &tm_k8, &k_full[ks], 0, krow, bh);
          } else {
            castdev::tma_load_3d(kd, &tm_k16, &k_full[ks], 0, krow, bh);
            castdev::tma_load_3d(kd + 16384, &tm_k16, &k_full[ks], 64, krow, bh);
          }
          issued = j + 1;
        }
        // Drain: every issued load completes before the CTA may exit.
        castdev::mbar_wait_drain(q_full, 0, err);
        for (int j = max(0, issued - KS); j < issued; ++j)
          castdev::mbar_wait_drain(&k_full[j % KS], (j / KS) & 1, err);
      }
    } else if (warp == kVProducerWarp) {
      // ---------------------------------------------------- V producer
      if (lane == 0 && n_kv > 0) {
        int issued = 0;
        for (int j = 0; j < n_kv; ++j) {  // ring position j
          const int kt = kt_lo + ring0.key_tile(j);
          const int blk = blist[kt / p.k_tiles];
          const int tin = kt % p.k_tiles;
          const bool blk_ok = blk >= 0 && blk < p.nkb;
          const int krow = blk_ok ? blk * p.k_block + tin * 128 : 0;
          const int vs = j % kVStages;
          if (j >= kVStages && !castdev::mbar_wait(&v_empty[vs], ((j / kVStages) - 1) & 1, err))
            break;
          uint8_t *vd = smem + v_off + vs * 32768;
          castdev::mbar_arrive_expect_tx(&v_full[vs], 32768);
          if (p.nkb_full > 0 && (!blk_ok || blk < p.nkb_full)) {
            // whole block (rows past its end are zeros), or an entry the
            // attention skips: a tile wholly outside the map, all zeros
            const int r = blk_ok ? tin * 128 : p.k_block;
            const int b = blk_ok ? blk : 0;
            castdev::tma_load_4d(vd, &tm_vb, &v_full[vs], 0, r, b, bh);
            castdev::tma_load_4d(vd + 16384, &tm_vb, &v_full[vs], 64, r, b, bh);
          } else {
            castdev::tma_load_3d(vd, &tm_v, &v_full[vs], 0, krow, bh);
            castdev::tma_load_3d(vd + 16384, &tm_v, &v_full[vs], 64, krow, bh);
          }
          issued = j + 1;
        }
        for (int j = max(0, issued - kVStages); j < issued; ++j)
          castdev::mbar_wait_drain(&v_full[j % kVStages], (j / kVStages) & 1, err);
      }
    } else {
      // ---------------------------------------------------- MMA issuers
      const int i = warp == kMmaWarp ? 0 : 1;
      if (lane == 0 && n_kv > 0 && i < n_groups) {
        const uint32_t sbase = castdev::smem_u32(smem);
        const RingMap ring{split ? 1 : 0, i, n_a, n_b};
        const int steps = 2 * (i == 0 ? n_a : n_b);
        if (mode)
          mma_issuer<1>(i, ring, tmem, sbase, steps, q_bytes, k_off, v_off, q_full, k_full,
                        k_empty, v_full, v_empty, s_full, p_full, pv_done, err);
        else
          mma_issuer<0>(i, ring, tmem, sbase, steps, q_bytes, k_off, v_off, q_full, k_full,
                        k_empty, v_full, v_empty, s_full, p_full, pv_done, err);
        // Every MMA this thread issued completes before TMEM is released.
        castdev::tc_commit(&mma_drain[i]);
        castdev::mbar_wait_drain(&mma_drain[i], 0, err);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int ti = warp >> 2;  // query tile handled by this warpgroup
    const int row = (warp & 3) * 32 + lane;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t o_addr = tmem + lane_off + ti * 128;
    const uint32_t s_addr = tmem + lane_off + 256 + ti * 128;
    const bool active = ti < n_groups;
    const int my_steps = 2 * (ti == 0 ? n_a : n_b);           // 64-key steps of this warpgroup
    const int start_tile = kt_lo + ((split && ti == 1) ? n_a : 0);  // its first key tile
    const int qrow_in_block = (t0 + (split ? 0 : ti)) * 128 + row;
    const int qrow = qb * p.q_block + qrow_in_block;
    const bool row_valid = active && qrow_in_block < p.q_block && qrow < p.Lq;
    const float qscale = mode ? p.q_scales[row_item] : 1.0f;
    float m_run = -INFINITY, l_run = 0.0f;
    bool ok = true;
    // The step loop, compiled once per QK^T precision so each copy holds only
    // its own code.
    auto run_steps = [&](auto int8_tag) {
      constexpr bool kInt8 = decltype(int8_tag)::value;
      // Per list entry: first key row, keys inside the block (clipped to Lk)
      // and the QK^T scale in log2 units (int8: q_scale * k_scale); the next
      // entry's values are fetched one entry ahead.
      struct Entry {
        int krow0, nvalid;
        float c2;
      };
      auto fetch = [&](int jb) {
        Entry e{0, 0, p.sm_scale_log2};
        if (jb < n_blocks) {
          const int blk = blist[jb];
          if (blk >= 0 && blk < p.nkb) {
            e.krow0 = blk * p.k_block;
            e.nvalid = min(p.k_block, p.Lk - e.krow0);
            if (kInt8) e.c2 *= qscale * p.k_scales[(size_t)bh * p.nkb + blk];
          }
        }
        return e;
      };
      int jb = start_tile / p.k_tiles;            // list entry
      int koff = (start_tile % p.k_tiles) * 128;  // key offset of this step inside it
      Entry cur = fetch(jb), nxt = fetch(jb + 1);
      const int block_keys = p.k_tiles * 128;
      for (int h = 0; h < my_steps; ++h) {
        const int half = h & 1;
        const float c2 = cur.c2;
        const int valid_cols = max(0, min(64, cur.nvalid - koff));
        const int krow = cur.krow0 + koff;
        // Key mask of this step: columns >= valid_cols, and key_valid == 0.
        uint32_t kmask[2];
#pragma unroll
        for (int w = 0; w < 2; ++w) {
          const int lo = valid_cols - 32 * w;
          kmask[w] = lo >= 32 ? 0xffffffffu : (lo <= 0 ? 0u : ((1u << lo) - 1u));
        }
        if (p.key_valid && valid_cols > 0) {
          // 16-byte loads for whole chunks inside the step's valid keys when
          // the step's first key is 16-byte aligned in key_valid (key blocks
          // of any size start anywhere), byte loads otherwise and for a
          // ragged last chunk; nothing past key valid_cols - 1.
          const uint8_t *kv = p.key_valid + krow;
          const bool kv16 = (reinterpret_cast<uintptr_t>(kv) & 15u) == 0;
#pragma unroll
          for (int w = 0; w < 2; ++w) {
            uint32_t bits = 0;
#pragma unroll
            for (int q2 = 0; q2 < 2; ++q2) {
              const int c0 = 32 * w + 16 * q2;
              uint32_t words[4] = {0u, 0u, 0u, 0u};
              if (kv16 && c0 + 16 <= valid_cols) {
                const uint4 b = *reinterpret_cast<const uint4 *>(kv + c0);
                words[0] = b.x, words[1] = b.y, words[2] = b.z, words[3] = b.w;
              } else if (c0 < valid_cols) {
                for (int c = c0; c < min(valid_cols, c0 + 16); ++c)
                  words[(c - c0) >> 2] |= (uint32_t)kv[c] << (8 * ((c - c0) & 3));
              }
#pragma unroll
              for (int q4 = 0; q4 < 4; ++q4)
#pragma unroll
                for (int by = 0; by < 4; ++by)
                  if ((words[q4] >> (8 * by)) & 0xFFu) bits |= 1u << (16 * q2 + 4 * q4 + by);
            }
            kmask[w] &= bits;
          }
        }
        const bool full_step = (kmask[0] & kmask[1]) == 0xffffffffu;

        ok = __all_sync(0xffffffffu, castdev::mbar_wait(&s_full[ti * 2 + half], (h >> 1) & 1, err));
        if (!ok) break;
        castdev::tc_fence_after();
        const uint32_t sb = s_addr + 64 * half;
        uint32_t v[64];
        castdev::tmem_ld32(sb, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
        castdev::tmem_ld32(sb + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
        castdev::tmem_wait_ld();

        // Fast path: exponentials against the running max in one pass.  A
        // step sum above kFastSumLimit (or no running max yet) sends the warp
        // to the exact path: true step max, lazy update of the running max,
        // rescale of O, exponentials again from S.
        float sum = 0.0f;
        bool slow = __any_sync(0xffffffffu, m_run == -INFINITY);
        if (!slow) {
          sum = step_probs_any<kInt8>(v, kmask, full_step, c2, m_run);
          slow = __any_sync(0xffffffffu, !(sum <= kFastSumLimit));
          if (slow) {
            castdev::tmem_ld32(sb, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
            castdev::tmem_ld32(sb + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
            castdev::tmem_wait_ld();
          }
        }
        if (__builtin_expect(slow, 0)) {
          const float m_step = full_step ? row_max<kInt8, false>(v, kmask, c2)
                                         : row_max<kInt8, true>(v, kmask, c2);
          float o_scale = 1.0f;
          if (m_step > m_run + kRescaleLog2 || m_run == -INFINITY) {
            const float m_new = fmaxf(m_run, m_step);
            o_scale = (m_run == -INFINITY) ? (m_new == -INFINITY ? 1.0f : 0.0f)
                                           : fast_exp2(m_run - m_new);
            l_run *= o_scale;
            m_run = m_new;
          }
          if (h > 0 && __any_sync(0xffffffffu, o_scale != 1.0f)) {
            // O_i += P_i(h-1) V_{h-1} may still be running.  Its barrier is
            // at most one phase behind: S_i(h), already waited for, was
            // committed after PV_i(h-2).
            const int hp = h - 1;
            ok = __all_sync(0xffffffffu,
                            castdev::mbar_wait(&pv_done[ti * 2 + (hp & 1)], (hp >> 1) & 1, err));
            if (!ok) break;
            castdev::tc_fence_after();
#pragma unroll 1
            for (int cc = 0; cc < 4; ++cc) {
              uint32_t o[32];
              castdev::tmem_ld32(o_addr + 32 * cc, o);
              castdev::tmem_wait_ld();
#pragma unroll
              for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * o_scale);
              castdev::tmem_st32(o_addr + 32 * cc, o);
            }
          }
          const float base = (m_run == -INFINITY) ? 0.0f : m_run;
          sum = step_probs_any<kInt8>(v, kmask, full_step, c2, base);
        }
        castdev::tmem_st32(sb, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
        l_run += sum;
        castdev::tmem_wait_st();
        castdev::tc_fence_before();
        __syncwarp();
        if (lane == 0) castdev::mbar_arrive(&p_full[ti * 2 + half]);
        koff += 64;
        if (koff == block_keys) {
          koff = 0;
          ++jb;
          cur = nxt;
          nxt = fetch(jb + 1);
        }
      }
    };
    if (active) {
      if (mode)
        run_steps(std::integral_constant<bool, true>{});
      else
        run_steps(std::integral_constant<bool, false>{});
    }
    // ------------------------------------------------------------ epilogue
    if (active && ok && my_steps > 0) {
      // the last PV's commit covers every earlier MMA of this tile
      const int hl = my_steps - 1;
      ok = __all_sync(0xffffffffu,
                      castdev::mbar_wait(&pv_done[ti * 2 + (hl & 1)], (hl >> 1) & 1, err));
      castdev::tc_fence_after();
    }
    if (split && ti == 1) {
      // Split item: leave this half's running max and row sum in the tile's
      // dead S columns for warpgroup 0, which merges O1 into its result.
      if (ok) {
        castdev::tmem_st1(s_addr, __float_as_uint(m_run));
        castdev::tmem_st1(s_addr + 1, __float_as_uint(l_run));
        castdev::tmem_wait_st();
      }
      castdev::tc_fence_before();
      __syncwarp();
      if (lane == 0) castdev::mbar_arrive(merge_bar);
    } else if (active) {
      float scale0 = 1.0f, scale1 = 0.0f;
      const uint32_t o1_addr = tmem + lane_off + 128;
      if (split && ok) {
        ok = __all_sync(0xffffffffu, castdev::mbar_wait(merge_bar, 0, err));
        castdev::tc_fence_after();
        const uint32_t s1_addr = tmem + lane_off + 256 + 128;
        const float m1 = __uint_as_float(castdev::tmem_ld1(s1_addr));
        const float l1 = __uint_as_float(castdev::tmem_ld1(s1_addr + 1));
        castdev::tmem_wait_ld();
        const float m = fmaxf(m_run, m1);
        scale0 = m == -INFINITY ? 0.0f : fast_exp2(m_run - m);
        scale1 = m == -INFINITY ? 0.0f : fast_exp2(m1 - m);
        l_run = l_run * scale0 + l1 * scale1;
        m_run = m;
      }
      // 32 columns of this row's O (the split halves merged), unnormalised
      auto load_o = [&](int cc, uint32_t (&o)[32]) {
        if (my_steps > 0) {
          castdev::tmem_ld32(o_addr + 32 * cc, o);
          if (split) {
            uint32_t o1[32];
            castdev::tmem_ld32(o1_addr + 32 * cc, o1);
            castdev::tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c)
              o[c] = __float_as_uint(fmaf(__uint_as_float(o1[c]), scale1,
                                          __uint_as_float(o[c]) * scale0));
          } else {
            castdev::tmem_wait_ld();
          }
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) o[c] = 0u;
        }
      };
      auto store_row = [&](int cc, const float (&o)[32], float inv_l) {
        uint4 w[4];
        uint32_t *wp = reinterpret_cast<uint32_t *>(w);
#pragma unroll
        for (int c = 0; c < 16; ++c) wp[c] = pack_bf16x2(o[2 * c] * inv_l, o[2 * c + 1] * inv_l);
        const size_t off = ((size_t)bh * p.Lq + qrow) * 128 + 32 * cc;
        uint4 *dst = reinterpret_cast<uint4 *>(p.out + off);
#pragma unroll
        for (int c = 0; c < 4; ++c) dst[c] = w[c];
        for (int r = 0; r < p.n_peers; ++r) {
          uint4 *pd = reinterpret_cast<uint4 *>(p.peer_out[r] + off);
#pragma unroll
          for (int c = 0; c < 4; ++c) pd[c] = w[c];
        }
      };
      if (n_live == 1) {
        // the whole item ran here: normalise and write
        if (ok) {
          const float inv_l = l_run > 0.0f ? 1.0f / l_run : 0.0f;
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            uint32_t o[32];
            load_o(cc, o);
            if (row_valid) store_row(cc, *reinterpret_cast<float(*)[32]>(o), inv_l);
          }
          if (row_valid && p.lse)
            p.lse[(size_t)bh * p.Lq + qrow] = l_run > 0.0f ? m_run + __log2f(l_run) : -INFINITY;
        }
      } else {
        // Cut item: leave this part's O, running max and row sum in its
        // slot; the item's last part to arrive merges every slot
        // (O = sum_j O_j 2^(m_j - m), l likewise, m = max_j m_j).
        const uint32_t n_thr = 128u * (split ? 1u : (uint32_t)nq);
        const int mo = 2 * 128 * 128 + ti * 256 + row;  // running max of this row in a slot
        float *slot = p.part_ws + (size_t)(blockIdx.x - p.n_whole) * kPartSlotFloats;
        if (ok) {
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            uint32_t o[32];
            load_o(cc, o);
            float *dst = slot + ti * 16384 + 32 * cc * 128 + row;
#pragma unroll
            for (int c = 0; c < 32; ++c) dst[c * 128] = __uint_as_float(o[c]);
          }
          slot[mo] = m_run;
          slot[mo + 128] = l_run;
        }
        __threadfence();
        castdev::named_bar_sync(1, n_thr);
        if (threadIdx.x == 0) {
          const int prev = atomicAdd(&p.part_counter[split_idx], 1);
          const uint32_t last = prev == n_live - 1;
          if (last) atomicExch(&p.part_counter[split_idx], 0);
          *part_flag = last;
          __threadfence();
        }
        castdev::named_bar_sync(1, n_thr);
        if (*part_flag) {
          const float *base = p.part_ws + (size_t)p.part_first[split_idx] * kPartSlotFloats;
          float m = -INFINITY;
          for (int j = 0; j < n_live; ++j) m = fmaxf(m, __ldcg(base + (size_t)j * kPartSlotFloats + mo));
          float l = 0.0f;
          for (int j = 0; j < n_live; ++j) {
            const float *sj = base + (size_t)j * kPartSlotFloats;
            const float mj = __ldcg(sj + mo);
            if (mj != -INFINITY) l = fmaf(__ldcg(sj + mo + 128), fast_exp2(mj - m), l);
          }
          const float inv_l = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll 1
          for (int cc = 0; cc < 4; ++cc) {
            float acc[32];
#pragma unroll
            for (int c = 0; c < 32; ++c) acc[c] = 0.0f;
            for (int j = 0; j < n_live; ++j) {
              const float *sj = base + (size_t)j * kPartSlotFloats;
              const float mj = __ldcg(sj + mo);
              const float w = mj == -INFINITY ? 0.0f : fast_exp2(mj - m);
              const float *oj = sj + ti * 16384 + 32 * cc * 128 + row;
#pragma unroll
              for (int c = 0; c < 32; ++c) acc[c] = fmaf(__ldcg(oj + c * 128), w, acc[c]);
            }
            if (row_valid) store_row(cc, acc, inv_l);
          }
          if (row_valid && p.lse)
            p.lse[(size_t)bh * p.Lq + qrow] = l > 0.0f ? m + __log2f(l) : -INFINITY;
        }
      }
    }
  }

  // this thread's output stores (peer ones included) before the ticket
  if (p.n_peers > 0) __threadfence_system();
  __syncthreads();
  if (warp == kMmaWarp) {
    castdev::tc_fence_after();
    castdev::tmem_dealloc(tmem, 512);
  }
  if (p.n_peers > 0 && threadIdx.x == 0) peer_ticket(p);
}

}  // namespace castk
