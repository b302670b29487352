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
  int min_count_flip;        // INT_MAX - the smallest count over every row (0: no row yet)
  int max_count;             // the largest count over every row
  int current_changed;       // a swap removed or added a current-chunk key
  int hist_delta;            // historical slots added minus removed by the swaps
  unsigned long long count_sum, hist_before;
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
                      float *__restrict__ err_out, int *__restrict__ limit_out, SwapCtl *ctl,
                      const int *__restrict__ gate) {
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
  if (gate && *gate) return;  // a transport gate failed: the call leaves the selection as it is
  // every row's count statistics (memory rows take no search, but their
  // swappable counts widen the candidate list): the grid strides over the
  // B*H*Q rows, one thread per row
  for (int qr = blockIdx.x * blockDim.x + tid; qr < p.B * p.H * p.Q; qr += gridDim.x * blockDim.x) {
    const long long c = __ldg(counts + qr);
    int sw = 0, hist = 0;
    for (int j = 0; j < p.S && j < c; ++j) {
      const bool h = __ldg(selected + (size_t)qr * p.S + j) < p.M;
      hist += h;
      sw += !p.historical || h;
    }
    if (sw) atomicMax(&ctl->max_swappable, sw);
    const int ci = (int)min(max(c, 0ll), (long long)INT_MAX);
    atomicMax(&ctl->min_count_flip, INT_MAX - ci);
    atomicMax(&ctl->max_count, ci);
    atomicAdd(&ctl->count_sum, (unsigned long long)max(c, 0ll));
    if (hist) atomicAdd(&ctl->hist_before, (unsigned long long)hist);
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
                      int search, int obj_slot, int finish, float swap_eps, int max_swaps,
                      const int *__restrict__ gate) {
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
  if (gate && *gate) {  // a transport gate failed: no work; the last CTA writes zero stats
    search = 0;
    obj_slot = -1;
    if (tid == 0) {
      __threadfence();
      last = atomicAdd(&ctl->ticket, 1u) == (unsigned)(gridDim.x - 1);
    }
    __syncthreads();
    if (last && tid == 0) {
      if (finish)
        for (int i = 0; i < 5; ++i) stats[i] = 0.0;
      if (finish)
        for (int i = 8; i < 14; ++i) stats[i] = 0.0;
      ctl->ticket = 0u;
    }
    return;
  }
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
          ctl->current_changed |= (k >= p.M) || (cg[b.l] >= p.M);
          ctl->hist_delta += (cg[b.l] < p.M ? 1 : 0) - (k < p.M ? 1 : 0);
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
      stats[8] = (double)(INT_MAX - ctl->min_count_flip);
      stats[9] = (double)ctl->max_count;
      stats[10] = (double)ctl->count_sum;
      stats[11] = (double)ctl->hist_before;
      stats[12] = (double)ctl->hist_before + (double)ctl->hist_delta;
      stats[13] = (double)ctl->current_changed;
    }
  }
  if (tid == 0) ctl->ticket = 0u;
}

// ---------------------------------------------------------------------------
// The routing objective on the device: transport operators, coefficient
// vector and Hessian over the current rows, and the transport gates.
// ---------------------------------------------------------------------------
constexpr int kSwapObjThreads = 256;
constexpr int kSwapObjMaxTargets = 32, kSwapObjMaxPairs = 16, kSwapObjMaxCells = 64;
constexpr int kSwapObjMaxBins = 2048;  // tiles x bins of one sketch (18 x 66 = 1188)

struct SwapObjTarget {
  const float *theta, *aff;  // the pair's sketch [tiles][bins], or NULL: identity operator
  float x_l, x_r;            // exponents of the left and right operators: a and -(1-a)
  float s_l, s_r;            // their weights: 1-a and a
  int lc, rc;                // left and right anchor cells
};

struct SwapObjPair {          // a same-segment anchor pair with skipped frames
  const float *mean;          // its sketch's mean affinity on the device, or NULL: mean_val
  float mean_val;
  int c_lo, c_hi;             // the cells of its skipped frames, inclusive
  int matching;               // it has a sketch (counts for the transport gate)
};

struct SwapObjParams {
  int n, tiles, bins, cells, R, T, n_pairs;
  const float *u_re, *u_im;   // [tiles][bins][n]
  const float *v_re, *v_im;   // [tiles][n][bins]
  float lam_a, lam_r, min_match, min_pair;
  int require_fc, pair_gate;
  float cell_count[kSwapObjMaxCells];
  SwapObjTarget t[kSwapObjMaxTargets];
  SwapObjPair pr[kSwapObjMaxPairs];
  float *ops;                 // [2T][n][n] (out, in), weighted
  float *coef, *hess;         // [R], [R][R]
  uint8_t *row_gate;          // [R] (pair gate) or NULL
  int *gate;                  // 0 ok, 1 weak transport, 2 no strong pair cells
  double *stats;              // [5]: gate, [6]: matching affinity, [7]: gated cells
};

// grid (2T, ceil(n*n / 8)), 8 warps: op k = 2t + side is
//   s * (I + sum_p V_p ((exp(i x g_p theta_p) - 1) * U_p))
// (side 0: x = a, s = 1-a; side 1: x = -(1-a), s = a).  Each warp computes
// one output entry (o, j), its lanes splitting the tiles x bins terms, then a
// shuffle reduction.  CTA (0, 0) also evaluates the transport gates.
__global__ void __launch_bounds__(kSwapObjThreads) swap_operator_kernel(const __grid_constant__ SwapObjParams p) {
  __shared__ float rc_[kSwapObjMaxBins], rs_[kSwapObjMaxBins];
  const int k = blockIdx.x, t = k >> 1, side = k & 1;
  const SwapObjTarget &tg = p.t[t];
  const float x = side ? tg.x_r : tg.x_l, sc = side ? tg.s_r : tg.s_l;
  const int nb = p.tiles * p.bins;
  if (tg.theta)
    for (int i = threadIdx.x; i < nb; i += blockDim.x) {
      const float ang = __fmul_rn(__fmul_rn(x, tg.aff[i]), tg.theta[i]);
      float sn, cs;
      sincosf(ang, &sn, &cs);
      rc_[i] = cs - 1.0f;
      rs_[i] = sn;
    }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int idx = blockIdx.y * (kSwapObjThreads / 32) + warp;
  if (idx < p.n * p.n) {
    const int o = idx / p.n, j = idx % p.n;
    float acc0 = 0.f, acc1 = 0.f;
    if (tg.theta)
      for (int i = lane; i < nb; i += 64) {
#pragma unroll
        for (int u2 = 0; u2 < 2; ++u2) {
          const int ii = i + 32 * u2;
          if (ii >= nb) break;
          const int tp = ii / p.bins, f = ii - tp * p.bins;
          const float a = __ldg(p.u_re + (size_t)ii * p.n + j), b = __ldg(p.u_im + (size_t)ii * p.n + j);
          const float vr = __ldg(p.v_re + ((size_t)tp * p.n + o) * p.bins + f);
          const float vi = __ldg(p.v_im + ((size_t)tp * p.n + o) * p.bins + f);
          const float c = rc_[ii], s = rs_[ii];
          const float wr = c * a - s * b, wi = c * b + s * a;
          if (u2 == 0)
            acc0 = fmaf(vr, wr, fmaf(vi, wi, acc0));
          else
            acc1 = fmaf(vr, wr, fmaf(vi, wi, acc1));
        }
      }
    float acc = acc0 + acc1;
    for (int off = 16; off; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) p.ops[(size_t)k * p.n * p.n + idx] = sc * ((o == j ? 1.f : 0.f) + acc);
  }
  if (k == 0 && blockIdx.y == 0 && threadIdx.x == 0) {
    int status = 0;
    float match = 0.f;
    bool any = false;
    for (int i = 0; i < p.n_pairs; ++i)
      if (p.pr[i].matching) {
        const float m = p.pr[i].mean ? *p.pr[i].mean : p.pr[i].mean_val;
        match = any ? fmaxf(match, m) : m;
        any = true;
      }
    if (p.require_fc && !(any && match >= p.min_match)) status = 1;
    int gated = 0;
    if (status == 0 && p.pair_gate) {
      bool cell[kSwapObjMaxCells] = {};
      for (int i = 0; i < p.n_pairs; ++i) {
        const float m = p.pr[i].mean ? *p.pr[i].mean : p.pr[i].mean_val;
        if (!(m >= p.min_pair)) continue;
        for (int c = p.pr[i].c_lo; c <= p.pr[i].c_hi; ++c) {
          gated += !cell[c];
          cell[c] = true;
        }
      }
      for (int r = 0; r < p.R; ++r) p.row_gate[r] = cell[r / p.n] ? 1 : 0;
      if (!gated) status = 2;
    }
    *p.gate = status;
    p.stats[5] = status;
    p.stats[6] = match;
    p.stats[7] = gated;
  }
}

// grid-stride over R*R + R: the Hessian, every entry summed over the
// targets in order (no atomics), then the anchor coefficients
//   hess[(ci,a),(cj,b)] = lam_r * sum_t sum_k X_t[k][a] Y_t[k][b]
// with X, Y the target's operator on the side of cell ci, cj (A + B when
// both anchors share a cell), and coef[(c,a)] = lam_a * anchors in cell c.
__global__ void __launch_bounds__(kSwapObjThreads) swap_hessian_kernel(const __grid_constant__ SwapObjParams p) {
  const int n = p.n, nn = n * n;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < p.R * p.R + p.R; i += gridDim.x * blockDim.x) {
    if (i >= p.R * p.R) {
      const int r = i - p.R * p.R;
      p.coef[r] = p.lam_a * p.cell_count[r / n];
      continue;
    }
    const int row = i / p.R, col = i % p.R;
    const int ci = row / n, a = row % n, cj = col / n, b = col % n;
    float acc = 0.f;
    for (int t = 0; t < p.T; ++t) {
      const SwapObjTarget &tg = p.t[t];
      const float *A = p.ops + (size_t)(2 * t) * nn, *B = A + nn;
      if (tg.lc == tg.rc) {
        if (ci != tg.lc || cj != tg.lc) continue;
        float s = 0.f;
        for (int kk = 0; kk < n; ++kk)
          s = fmaf(A[kk * n + a] + B[kk * n + a], A[kk * n + b] + B[kk * n + b], s);
        acc += s;
      } else {
        const float *X = ci == tg.lc ? A : (ci == tg.rc ? B : nullptr);
        const float *Y = cj == tg.lc ? A : (cj == tg.rc ? B : nullptr);
        if (!X || !Y) continue;
        float s = 0.f;
        for (int kk = 0; kk < n; ++kk) s = fmaf(X[kk * n + a], Y[kk * n + b], s);
        acc += s;
      }
    }
    p.hess[i] = p.lam_r * acc;
  }
}

}  // namespace castk
