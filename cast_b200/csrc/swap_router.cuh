// FC-PASM fixed-budget swap router: omission proxies and single-swap
// coordinate-descent rounds over the current rows of a pooled block score.
//
// Replaces the numeric body of FCPASMLocalCoordinateSwapRouter.refine
// (proposed/fc_pasm_swap_routing.py:616-1077): candidates (:838-845), the
// omission proxy (estimate_block_omission_error :64-106), the row errors
// (:870-871), the quadratic terms (_objective_terms :414-548) and the swap
// search with its one global argmin per round (:894-990).  The objective is
// written as J(e) = sum_r c_r |e_r|^2 + e^T H e over the current rows, c and
// H built by the caller from the transport operators, so a round needs only
// a_r = c_r + H_rr and b_r = (H e)_r - H_rr e_r per row.
//
// Work is tiny and latency-bound (a few thousand pooled rows): one CTA per
// (batch, head, current row) for the proxies, one CTA per (batch, head) per
// round, and the last CTA of a round (atomic ticket) reduces the per-head
// bests in (batch, head, row) order and applies the swap, so a whole call is
// 2 + rounds launches with no host synchronisation.
#pragma once

#include "common.cuh"

namespace castk {

constexpr int kSwapProxyThreads = 128;
constexpr int kSwapRoundThreads = 256;

struct SwapShape {
  int B, H, Q, K, D, S, M, R, Lc, G, cand_blocks, mult, historical, same_bank;
};

// Call-wide state in the workspace; zeroed by the proxy launch.
struct SwapCtl {
  unsigned int ticket;
  int swaps;
  double improvement;
};

// Per (batch, head) best pair of a round.
struct SwapBest {
  float value;
  int row, s, l;
};

__device__ __forceinline__ bool swap_better(float v, long long key, float bv, long long bkey) {
  return v < bv || (v == bv && key < bkey);
}

__device__ __forceinline__ float block_reduce_max(float v, float *red) {
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float r = red[0];
  for (int i = 1; i < nw; ++i) r = fmaxf(r, red[i]);
  return r;
}

__device__ __forceinline__ float block_reduce_sum(float v, float *red) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float r = 0.f;
  for (int i = 0; i < nw; ++i) r += red[i];
  return r;
}

// One CTA per current row (b, h, r): the row's softmax, its pooled output
// P.V, the top-Lc candidates of score + 1e6*local (larger first, lower index
// on ties), the proxies scale*(out - V[c]) averaged over G sketch groups
// (scale = p/(1-p+eps)), the row's candidate limit and its error: the sum of
// the proxies of valid candidates that are not already selected.
__global__ void __launch_bounds__(kSwapProxyThreads)
    swap_proxy_kernel(const float *__restrict__ score, const float *__restrict__ value,
                      const long long *__restrict__ selected, const long long *__restrict__ counts,
                      const uint8_t *__restrict__ local, SwapShape p, float eps,
                      int *__restrict__ cand_out, float *__restrict__ proxy_out,
                      float *__restrict__ err_out, int *__restrict__ limit_out, SwapCtl *ctl) {
  extern __shared__ float sm[];
  float *prob = sm;                 // K
  float *rk = prob + p.K;           // K
  float *outv = rk + p.K;           // D
  float *red = outv + p.D;          // 32
  int *cand = reinterpret_cast<int *>(red + 32);  // Lc
  int *kept = cand + p.Lc;          // Lc
  int *seli = kept + p.Lc;          // S
  const int row = blockIdx.x;
  const int bh = row / p.R, r = row % p.R, q = p.M + r;
  const int tid = threadIdx.x;
  if (row == 0 && tid == 0) {
    ctl->ticket = 0u;
    ctl->swaps = 0;
    ctl->improvement = 0.0;
  }
  const float *srow = score + ((size_t)bh * p.Q + q) * p.K;
  const float *V = value + (size_t)bh * p.K * p.D;
  const uint8_t *lrow = local + (size_t)q * p.K;

  float m = -INFINITY;
  for (int k = tid; k < p.K; k += blockDim.x) m = fmaxf(m, __ldg(srow + k));
  m = block_reduce_max(m, red);
  float s = 0.f;
  for (int k = tid; k < p.K; k += blockDim.x) {
    const float e = expf(__ldg(srow + k) - m);
    prob[k] = e;
    s += e;
  }
  s = block_reduce_sum(s, red);
  for (int k = tid; k < p.K; k += blockDim.x) {
    prob[k] = prob[k] / s;
    if (k < p.cand_blocks) rk[k] = __fadd_rn(__ldg(srow + k), lrow[k] ? 1e6f : 0.f);
  }
  const long long cnt = __ldg(counts + (size_t)bh * p.Q + q);
  for (int j = tid; j < p.S; j += blockDim.x) seli[j] = (int)__ldg(selected + ((size_t)bh * p.Q + q) * p.S + j);
  // a NaN score leaves ranks unfilled: they name block 0 instead of garbage
  for (int l = tid; l < p.Lc; l += blockDim.x) cand[l] = 0;
  __syncthreads();

  for (int d = tid; d < p.D; d += blockDim.x) {
    float acc = 0.f;
    for (int k = 0; k < p.K; ++k) acc = fmaf(prob[k], __ldg(V + (size_t)k * p.D + d), acc);
    outv[d] = acc;
  }
  // rank of every candidate block by (ranking desc, index asc)
  for (int k = tid; k < p.cand_blocks; k += blockDim.x) {
    const float x = rk[k];
    int rank = 0;
    for (int j = 0; j < p.cand_blocks; ++j) {
      const float y = rk[j];
      rank += (y > x) || (y == x && j < k);
    }
    if (rank < p.Lc) cand[rank] = k;
  }
  __syncthreads();
  int swappable = 0;
  for (int j = 0; j < p.S; ++j)
    swappable += (j < cnt) && (!p.historical || seli[j] < p.M);
  const int limit = min(swappable * p.mult, p.cand_blocks);
  for (int l = tid; l < p.Lc; l += blockDim.x) {
    int hit = 0;
    for (int j = 0; j < p.S; ++j) hit |= (j < cnt) && (seli[j] == cand[l]);
    kept[l] = hit;
  }
  const int width = p.D / p.G;
  float *prow = proxy_out + (size_t)row * p.Lc * p.G;
  for (int i = tid; i < p.Lc * p.G; i += blockDim.x) {
    const int l = i / p.G, g = i % p.G;
    const int c = cand[l];
    const float pc = prob[c];
    const float scale = __fdiv_rn(pc, __fadd_rn(__fsub_rn(1.f, pc), eps));
    const float *vc = V + (size_t)c * p.D + g * width;
    float acc = 0.f;
    for (int t = 0; t < width; ++t)
      acc = __fadd_rn(acc, __fmul_rn(scale, __fsub_rn(outv[g * width + t], __ldg(vc + t))));
    prow[i] = __fdiv_rn(acc, (float)width);
  }
  for (int l = tid; l < p.Lc; l += blockDim.x) cand_out[(size_t)row * p.Lc + l] = cand[l];
  if (tid == 0) limit_out[row] = limit;
  __syncthreads();
  for (int g = tid; g < p.G; g += blockDim.x) {
    float e = 0.f;
    for (int l = 0; l < limit; ++l)
      if (!kept[l]) e += prow[l * p.G + g];
    err_out[(size_t)row * p.G + g] = e;
  }
}

// One CTA per (b, h).  Builds H e for the head's current-row errors, adds
// the head's objective to obj_part[obj_slot] (when obj_slot >= 0) and, when
// `search`, finds the head's best admissible (remove slot, add candidate)
// pair.  The last CTA to finish takes the first minimum over (b, h, row) and,
// if it beats -swap_eps and the swap cap allows, writes the added key into
// the selection and moves the row's error by (removed proxy - added proxy).
// With `finish` the last CTA writes the call's stats.
__global__ void __launch_bounds__(kSwapRoundThreads)
    swap_round_kernel(long long *__restrict__ selected, const long long *__restrict__ counts,
                      const uint8_t *__restrict__ local, const uint8_t *__restrict__ row_gate,
                      const float *__restrict__ coef, const float *__restrict__ hess, SwapShape p,
                      const int *__restrict__ cand_all, const float *__restrict__ proxy_all,
                      float *__restrict__ err_all, const int *__restrict__ limit_all, SwapBest *best_bh,
                      double *__restrict__ obj_part, SwapCtl *ctl, double *__restrict__ stats,
                      int search, int obj_slot, int finish, float swap_eps, int max_swaps) {
  extern __shared__ float sm[];
  const int RG = p.R * p.G;
  float *e = sm;            // R*G
  float *he = e + RG;       // R*G
  __shared__ double dred[kSwapRoundThreads / 32];
  __shared__ SwapBest wbest[kSwapRoundThreads / 32];
  __shared__ bool last;
  const int bh = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = blockDim.x >> 5;
  float *eg = err_all + (size_t)bh * RG;
  for (int i = tid; i < RG; i += blockDim.x) e[i] = eg[i];
  __syncthreads();
  double part = 0.0;
  for (int i = tid; i < RG; i += blockDim.x) {
    const int r = i / p.G, g = i % p.G;
    float acc = 0.f;
    for (int t = 0; t < p.R; ++t) acc = fmaf(__ldg(hess + (size_t)r * p.R + t), e[t * p.G + g], acc);
    he[i] = acc;
    part += (double)__ldg(coef + r) * e[i] * e[i] + (double)e[i] * acc;
  }
  for (int o = 16; o; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  if (lane == 0) dred[warp] = part;
  __syncthreads();
  if (tid == 0 && obj_slot >= 0) {
    double t = 0.0;
    for (int w = 0; w < nwarps; ++w) t += dred[w];
    obj_part[(size_t)obj_slot * p.B * p.H + bh] = t;
  }

  if (search) {
    SwapBest mine{INFINITY, 0, 0, 0};
    long long mkey = LLONG_MAX;
    for (int r = warp; r < p.R; r += nwarps) {
      if (row_gate && !row_gate[r]) continue;
      const int q = p.M + r;
      const size_t qrow = (size_t)bh * p.Q + q;
      const int *cand = cand_all + ((size_t)bh * p.R + r) * p.Lc;
      const float *prx = proxy_all + ((size_t)bh * p.R + r) * p.Lc * p.G;
      const long long cnt = __ldg(counts + qrow);
      const int limit = limit_all[(size_t)bh * p.R + r];
      const float hrr = __ldg(hess + (size_t)r * p.R + r);
      const float a = __ldg(coef + r) + hrr;
      for (int pi = lane; pi < p.S * p.Lc; pi += 32) {
        const int sl = pi / p.Lc, l = pi % p.Lc;
        const int key = (int)selected[qrow * p.S + sl];
        const int add = cand[l];
        if (sl < cnt && (key < 0 || key >= p.K)) {  // a selected key outside the score
          atomicExch(&g_cast_device_error, (int)CAST_ERR_INVALID_ARGUMENT);
          continue;
        }
        bool ok = sl < cnt && l < limit && !local[(size_t)q * p.K + key];
        if (p.historical) ok = ok && key < p.M;
        if (p.same_bank) ok = ok && ((key < p.M) == (add < p.M));
        if (!ok) continue;
        // addable: the candidate is not among the valid selected keys
        bool kept = false;
        for (int j = 0; j < cnt && j < p.S; ++j) kept |= (int)selected[qrow * p.S + j] == add;
        if (kept) continue;
        int lr = -1;  // the removed key's candidate slot (its proxy), if any
        for (int t = 0; t < p.Lc; ++t)
          if (cand[t] == key) { lr = t; break; }
        float v = 0.f;
        for (int g = 0; g < p.G; ++g) {
          const float eo = e[r * p.G + g];
          const float b = he[r * p.G + g] - hrr * eo;
          const float d = (lr >= 0 ? prx[lr * p.G + g] : 0.f) - prx[l * p.G + g];
          v += a * (2.f * eo * d + d * d) + 2.f * b * d;
        }
        const long long k2 = (long long)r * p.S * p.Lc + pi;
        if (swap_better(v, k2, mine.value, mkey)) {
          mine = SwapBest{v, r, sl, l};
          mkey = k2;
        }
      }
    }
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, mine.value, o);
      const long long ok2 = __shfl_xor_sync(0xffffffffu, mkey, o);
      const int orow = __shfl_xor_sync(0xffffffffu, mine.row, o);
      const int os = __shfl_xor_sync(0xffffffffu, mine.s, o);
      const int ol = __shfl_xor_sync(0xffffffffu, mine.l, o);
      if (swap_better(ov, ok2, mine.value, mkey)) {
        mine = SwapBest{ov, orow, os, ol};
        mkey = ok2;
      }
    }
    if (lane == 0) wbest[warp] = mine;
    __syncthreads();
    if (tid == 0) {
      SwapBest b = wbest[0];
      for (int w = 1; w < nwarps; ++w) {
        const SwapBest c = wbest[w];
        const long long kc = ((long long)c.row * p.S + c.s) * p.Lc + c.l;
        const long long kb = ((long long)b.row * p.S + b.s) * p.Lc + b.l;
        if (swap_better(c.value, kc, b.value, kb)) b = c;
      }
      best_bh[bh] = b;
    }
  }
  if (tid == 0) {
    __threadfence();
    last = atomicAdd(&ctl->ticket, 1u) == (unsigned)(gridDim.x - 1);
  }
  __syncthreads();
  if (!last || tid != 0) return;
  __threadfence();
  ctl->ticket = 0u;
  if (search) {
    int bb = -1;
    SwapBest b{INFINITY, 0, 0, 0};
    for (int i = 0; i < (int)gridDim.x; ++i) {
      const SwapBest c = best_bh[i];
      if (c.value < b.value) {  // first minimum in (b, h, row) order
        b = c;
        bb = i;
      }
    }
    const bool capped = max_swaps > 0 && ctl->swaps >= max_swaps;
    if (bb >= 0 && b.value < -swap_eps && !capped) {
      const size_t qrow = (size_t)bb * p.Q + p.M + b.row;
      const int *cand = cand_all + ((size_t)bb * p.R + b.row) * p.Lc;
      const float *prx = proxy_all + ((size_t)bb * p.R + b.row) * p.Lc * p.G;
      const int key = (int)selected[qrow * p.S + b.s];
      int lr = -1;
      for (int t = 0; t < p.Lc; ++t)
        if (cand[t] == key) { lr = t; break; }
      float *er = err_all + ((size_t)bb * p.R + b.row) * p.G;
      for (int g = 0; g < p.G; ++g)
        er[g] += (lr >= 0 ? prx[lr * p.G + g] : 0.f) - prx[b.l * p.G + g];
      selected[qrow * p.S + b.s] = cand[b.l];
      ctl->swaps += 1;
      ctl->improvement += -(double)b.value;
    }
  }
  if (finish) {
    const int BH = p.B * p.H;
    double before = 0.0, after = 0.0;
    for (int i = 0; i < BH; ++i) {
      before += obj_part[i];
      after += obj_part[BH + i];
    }
    stats[0] = (double)ctl->swaps;
    stats[1] = before;
    stats[2] = after;
    stats[3] = ctl->improvement;
  }
}

}  // namespace castk
