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
// (batch, head, current row) for the proxies and again for each round, and
// the last CTA of a round (atomic ticket) reduces the per-row bests in
// (batch, head, row) order and applies the swap, so a whole call is
// 2 + rounds launches with no host synchronisation.
#pragma once

#include "common.cuh"

namespace castk {

constexpr int kSwapProxyThreads = 128;
constexpr int kSwapRoundThreads = 128;

struct SwapShape {
  int B, H, Q, K, D, S, M, R, Lc, G, cand_blocks, mult, historical, same_bank;
  int stage_v;  // the head's pooled values fit in shared memory (16-byte loads)
};

// Call-wide state in the workspace; zeroed by the host before the proxy
// launch.  max_swappable is the largest swappable count over every row
// (memory rows included), which sets the reference's candidate width
// maximum_l = min(cand_blocks, mult * max_swappable).
struct SwapCtl {
  unsigned int ticket;
  int swaps;
  double improvement;
  int max_swappable;
};

// The reference's maximum_l: candidate slots at or beyond it hold no proxy
// (its candidate list is only that wide).
__device__ __forceinline__ int swap_width(const SwapShape &p, const SwapCtl *ctl) {
  return min(p.Lc, min(p.cand_blocks, p.mult * *(volatile const int *)&ctl->max_swappable));
}

// Per-row best pair of a round.
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
  float *vsm = sm;                  // K*D when staged, first so it is 16-byte aligned
  float *prob = sm + (p.stage_v ? p.K * p.D : 0);  // K
  float *rk = prob + p.K;           // K
  float *outv = rk + p.K;           // D
  float *red = outv + p.D;          // 32
  int *cand = reinterpret_cast<int *>(red + 32);  // Lc
  int *kept = cand + p.Lc;          // Lc
  int *seli = kept + p.Lc;          // S
  float *pxs = reinterpret_cast<float *>(seli + p.S);  // Lc*G
  const int row = blockIdx.x;
  const int bh = row / p.R, r = row % p.R, q = p.M + r;
  const int tid = threadIdx.x;
  // memory rows take no search but their swappable counts widen the
  // candidate list: the grid strides over them, one thread per row
  for (int mr = blockIdx.x * blockDim.x + tid; mr < p.B * p.H * p.M; mr += gridDim.x * blockDim.x) {
    const size_t qrow = (size_t)(mr / p.M) * p.Q + mr % p.M;
    const long long c = __ldg(counts + qrow);
    int sw = 0;
    for (int j = 0; j < p.S && j < c; ++j)
      sw += !p.historical || __ldg(selected + qrow * p.S + j) < p.M;
    if (sw) atomicMax(&ctl->max_swappable, sw);
  }
  const float *srow = score + ((size_t)bh * p.Q + q) * p.K;
  const float *Vg = value + (size_t)bh * p.K * p.D;
  const uint8_t *lrow = local + (size_t)q * p.K;
  if (p.stage_v)
    for (int i = tid; i < p.K * p.D / 4; i += blockDim.x)
      reinterpret_cast<float4 *>(vsm)[i] = __ldg(reinterpret_cast<const float4 *>(Vg) + i);
  const float *V = p.stage_v ? vsm : Vg;  // staged copy (visible after the next barrier)

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
#pragma unroll 8
    for (int k = 0; k < p.K; ++k) acc = fmaf(prob[k], V[(size_t)k * p.D + d], acc);
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
  if (tid == 0 && swappable) atomicMax(&ctl->max_swappable, swappable);
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
#pragma unroll 4
    for (int t = 0; t < width; ++t)
      acc = __fadd_rn(acc, __fmul_rn(scale, __fsub_rn(outv[g * width + t], vc[t])));
    const float v = __fdiv_rn(acc, (float)width);
    pxs[i] = v;
    prow[i] = v;
  }
  for (int l = tid; l < p.Lc; l += blockDim.x) cand_out[(size_t)row * p.Lc + l] = cand[l];
  if (tid == 0) limit_out[row] = limit;
  __syncthreads();
  for (int g = tid; g < p.G; g += blockDim.x) {
    float e = 0.f;
    for (int l = 0; l < limit; ++l)
      if (!kept[l]) e += pxs[l * p.G + g];
    err_out[(size_t)row * p.G + g] = e;
  }
}

// One CTA per current row (b, h, r).  Builds (H e)_r from the head's
// current-row errors, stores the row's objective term in obj_part[obj_slot]
// (when obj_slot >= 0) and, when `search`, the row's best admissible
// (remove slot, add candidate) pair, from per-row tables in shared memory.
// The last CTA to finish takes the first minimum over (b, h, row) with all
// its threads and, if it beats -swap_eps and the swap cap allows, writes the
// added key into the selection and moves the row's error by (removed proxy -
// added proxy).  With `finish` the last CTA writes the call's stats.
__global__ void __launch_bounds__(kSwapRoundThreads)
    swap_round_kernel(long long *__restrict__ selected, const long long *__restrict__ counts,
                      const uint8_t *__restrict__ local, const uint8_t *__restrict__ row_gate,
                      const float *__restrict__ coef, const float *__restrict__ hess, SwapShape p,
                      const int *__restrict__ cand_all, const float *__restrict__ proxy_all,
                      float *__restrict__ err_all, const int *__restrict__ limit_all, SwapBest *best_row,
                      double *__restrict__ obj_part, SwapCtl *ctl, double *__restrict__ stats,
                      int search, int obj_slot, int finish, float swap_eps, int max_swaps) {
  extern __shared__ float sm[];
  float *e = sm;                        // R*G: the head's current-row errors
  float *prx = e + p.R * p.G;           // Lc*G: this row's proxies
  float *rem = prx + p.Lc * p.G;        // S*G: proxy of each selected slot's key
  float *he = rem + p.S * p.G;          // G
  int *cand = reinterpret_cast<int *>(he + p.G);  // Lc
  int *addok = cand + p.Lc;             // Lc
  int *remok = addok + p.Lc;            // S
  int *key = remok + p.S;               // S
  float *hrow = reinterpret_cast<float *>(key + p.S);  // R: this row of H
  __shared__ double dred[kSwapRoundThreads / 32];
  __shared__ float vred[kSwapRoundThreads / 32];
  __shared__ long long kred[kSwapRoundThreads / 32];
  __shared__ bool last;
  const int row = blockIdx.x, bh = row / p.R, r = row % p.R, q = p.M + r;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int RG = p.R * p.G;
  const float *eg = err_all + (size_t)bh * RG;
  for (int i = tid; i < RG; i += blockDim.x) e[i] = eg[i];
  for (int t = tid; t < p.R; t += blockDim.x) hrow[t] = __ldg(hess + (size_t)r * p.R + t);
  __syncthreads();
  const float hrr = hrow[r];
  double part = 0.0;
  for (int g = tid; g < p.G; g += blockDim.x) {
    float acc = 0.f;
    for (int t = 0; t < p.R; ++t) acc = fmaf(hrow[t], e[t * p.G + g], acc);
    he[g] = acc;
    const float er = e[r * p.G + g];
    part += (double)__ldg(coef + r) * er * er + (double)er * acc;
  }
  for (int o = 16; o; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  if (lane == 0) dred[warp] = part;

  float best = INFINITY;
  long long bkey = LLONG_MAX;
  const bool gated = row_gate && !row_gate[r];
  if (search && !gated) {
    const size_t qrow = (size_t)bh * p.Q + q;
    const long long cnt = __ldg(counts + qrow);
    const int limit = limit_all[row];
    const int width = swap_width(p, ctl);
    const int *cg = cand_all + (size_t)row * p.Lc;
    const float *pg = proxy_all + (size_t)row * p.Lc * p.G;
    for (int i = tid; i < p.Lc * p.G; i += blockDim.x) prx[i] = pg[i];
    for (int l = tid; l < p.Lc; l += blockDim.x) cand[l] = cg[l];
    for (int j = tid; j < p.S; j += blockDim.x) key[j] = (int)selected[qrow * p.S + j];
    __syncthreads();
    for (int l = tid; l < p.Lc; l += blockDim.x) {
      bool kept = false;
      for (int j = 0; j < cnt && j < p.S; ++j) kept |= key[j] == cand[l];
      addok[l] = l < limit && !kept;
    }
    for (int j = tid; j < p.S; j += blockDim.x) {
      const int k = key[j];
      bool ok = j < cnt;
      if (ok && (k < 0 || k >= p.K)) {  // a selected key outside the score
        atomicExch(&g_cast_device_error, (int)CAST_ERR_INVALID_ARGUMENT);
        ok = false;
      }
      ok = ok && !local[(size_t)q * p.K + k];
      if (p.historical) ok = ok && k < p.M;
      remok[j] = ok;
      int lr = -1;  // the removed key's candidate slot (its proxy), if any
      for (int t = 0; t < width; ++t)
        if (cand[t] == k) { lr = t; break; }
      for (int g = 0; g < p.G; ++g) rem[j * p.G + g] = lr >= 0 ? prx[lr * p.G + g] : 0.f;
    }
    __syncthreads();
    const float a = __ldg(coef + r) + hrr;
    for (int pi = tid; pi < p.S * p.Lc; pi += blockDim.x) {
      const int sl = pi / p.Lc, l = pi % p.Lc;
      if (!remok[sl] || !addok[l]) continue;
      if (p.same_bank && ((key[sl] < p.M) != (cand[l] < p.M))) continue;
      float v = 0.f;
      for (int g = 0; g < p.G; ++g) {
        const float eo = e[r * p.G + g];
        const float b = he[g] - hrr * eo;
        const float d = rem[sl * p.G + g] - prx[l * p.G + g];
        v += a * (2.f * eo * d + d * d) + 2.f * b * d;
      }
      if (swap_better(v, pi, best, bkey)) {
        best = v;
        bkey = pi;
      }
    }
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const long long ok2 = __shfl_xor_sync(0xffffffffu, bkey, o);
      if (swap_better(ov, ok2, best, bkey)) {
        best = ov;
        bkey = ok2;
      }
    }
    if (lane == 0) {
      vred[warp] = best;
      kred[warp] = bkey;
    }
  }
  __syncthreads();
  if (tid == 0) {
    if (obj_slot >= 0) {
      double t = 0.0;
      for (int w = 0; w < nwarps; ++w) t += dred[w];
      obj_part[(size_t)obj_slot * gridDim.x + row] = t;
    }
    if (search) {
      SwapBest b{INFINITY, r, 0, 0};
      if (!gated) {
        float bv = vred[0];
        long long bk = kred[0];
        for (int w = 1; w < nwarps; ++w)
          if (swap_better(vred[w], kred[w], bv, bk)) bv = vred[w], bk = kred[w];
        if (bk != LLONG_MAX) b = SwapBest{bv, r, (int)(bk / p.Lc), (int)(bk % p.Lc)};
      }
      best_row[row] = b;
    }
    __threadfence();
    last = atomicAdd(&ctl->ticket, 1u) == (unsigned)(gridDim.x - 1);
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  const int n = gridDim.x;
  if (search) {
    // first minimum over (b, h, row): value, then row index
    float bv = INFINITY;
    long long bi = LLONG_MAX;
    for (int i = tid; i < n; i += blockDim.x) {
      const float v = best_row[i].value;
      if (swap_better(v, i, bv, bi)) bv = v, bi = i;
    }
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const long long oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (swap_better(ov, oi, bv, bi)) bv = ov, bi = oi;
    }
    if (lane == 0) vred[warp] = bv, kred[warp] = bi;
    __syncthreads();
    if (warp == 0) {  // the whole warp applies the swap: parallel scans, no serial loads
      for (int w = 1; w < nwarps; ++w)
        if (swap_better(vred[w], kred[w], bv, bi)) bv = vred[w], bi = kred[w];
      const bool capped = max_swaps > 0 && ctl->swaps >= max_swaps;
      if (bi != LLONG_MAX && bv < -swap_eps && !capped) {
        const SwapBest b = best_row[bi];
        const int bb = (int)(bi / p.R);
        const size_t qrow = (size_t)bb * p.Q + p.M + b.row;
        const int *cg = cand_all + (size_t)bi * p.Lc;
        const float *pg = proxy_all + (size_t)bi * p.Lc * p.G;
        const int k = (int)selected[qrow * p.S + b.s];
        const int width = swap_width(p, ctl);
        int lr = width;  // first candidate slot holding the removed key
        for (int t0 = 0; t0 < width; t0 += 32) {
          const int t = t0 + lane;
          const unsigned m = __ballot_sync(0xffffffffu, t < width && cg[t] == k);
          if (m) {
            lr = t0 + __ffs(m) - 1;
            break;
          }
        }
        float *er = err_all + (size_t)bi * p.G;
        for (int g = lane; g < p.G; g += 32)
          er[g] += (lr < width ? pg[lr * p.G + g] : 0.f) - pg[b.l * p.G + g];
        __syncwarp();
        if (lane == 0) {
          selected[qrow * p.S + b.s] = cg[b.l];
          ctl->swaps += 1;
          ctl->improvement += -(double)bv;
        }
      }
    }
  }
  if (finish) {
    double before = 0.0, after = 0.0;
    for (int i = tid; i < n; i += blockDim.x) before += obj_part[i], after += obj_part[n + i];
    for (int o = 16; o; o >>= 1) {
      before += __shfl_xor_sync(0xffffffffu, before, o);
      after += __shfl_xor_sync(0xffffffffu, after, o);
    }
    __syncthreads();
    if (lane == 0) dred[warp] = before;
    __syncthreads();
    if (tid == 0) {
      double t = 0.0;
      for (int w = 0; w < nwarps; ++w) t += dred[w];
      stats[1] = t;
    }
    __syncthreads();
    if (lane == 0) dred[warp] = after;
    __syncthreads();
    if (tid == 0) {
      double t = 0.0;
      for (int w = 0; w < nwarps; ++w) t += dred[w];
      stats[0] = (double)ctl->swaps;
      stats[2] = t;
      stats[3] = ctl->improvement;
      stats[4] = (double)ctl->max_swappable;
    }
  }
  if (tid == 0) ctl->ticket = 0u;
}

}  // namespace castk
