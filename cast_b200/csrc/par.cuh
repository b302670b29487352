// Phase-Aware Reconstruction (FC-PASM reference numerics) for sm_100a.
//
// Restates proposed/matrix_world_spectral_residual.py:2771-3662 with the
// factory knobs.  The 11x10 tile transforms are small direct real DFTs done in
// registers (one thread per channel); nothing here is GEMM-shaped.
//
//   par_stats_kernel     grid (chunk, tile, pair): windowed reflect-padded
//                        anchor tiles -> rfft2 -> per-chunk channel sums of
//                        R*conj(L) and |R*conj(L)|            (reads anchors)
//   par_finalize_kernel  grid (tile, pair): chunk sums -> coherence, base
//                        confidence, theta, PHAT displacement, ramp
//                        confidence, affinity g, mix weights per target
//   par_predict_kernel   grid (chunk, tile, pair): anchor spectra again,
//                        phase mix per target, irfft2, analysis window ->
//                        predicted windowed tiles (workspace)
//   par_ola_kernel       grid (pixel, target): normalised overlap-add, bf16
//                        write of the target frame                (writes)
//
// Tensor-core prediction (used when C % 8 == 0 and a pair has at most
// kParMmaTargets targets): the whole per-tile chain analysis window -> rfft2
// -> per-frequency mix -> irfft2 -> synthesis window is linear in the two
// anchor tiles and circular in the pixel offset, so a target's predicted
// tile is pred = F_L l + F_R r with F[p][q] = win[p] win[q] kern[(p - q) mod
// (11, 10)] and kern[d] = (1/110) sum_f c_kx Re(w_f e^{i w_f . d}) (c_kx = 1
// for kx = 0, 5, else 2: the c2r rows).
//   par_filter_kernel    grid (tile, target): kern for L and R from the mix
//                        weights, then F as bf16 hi + lo (the pair carries
//                        ~16 significant bits) in the shared-memory image
//                        the MMA reads
//   par_predict_mma_kernel grid (128-channel chunk, tile, pair): the anchor
//                        pixels of the tile gathered by TMA (one 64-channel
//                        row per load; reflect padding is in the row index),
//                        D[128 ch x 112 px] = A[128 ch x 224 (L|R px)] F via
//                        tcgen05.mma (A MN-major, F K-major, fp32 in TMEM),
//                        then the predicted tiles to the workspace
#pragma once

#include "common.cuh"

namespace castk {

constexpr int kParTH = 11, kParTW = 10, kParWF = 6;
constexpr int kParFreq = kParTH * kParWF;  // 66
constexpr int kParPix = kParTH * kParTW;   // 110
constexpr int kParGH = 3, kParGW = 6, kParTiles = kParGH * kParGW;
constexpr int kParPadH = 4, kParPadW = 5, kParStride = 8;
constexpr int kParH = 22, kParW = 40;
constexpr int kParChunk = 64;             // channels per CTA (one per thread)
constexpr int kParPartial = 3 * kParFreq;  // re, im of sum R*conj(L); sum |R*conj(L)|
constexpr int kParMaxTargets = 16;
constexpr int kParMaxPairs = 16;

struct ParTables {
  float win[kParPix];     // sqrt-Hann 11x10 (row-major)
  float cw[kParTW];       // cos(2*pi*k/10)
  float sw[kParTW];       // sin(2*pi*k/10)
  float ch[kParTH];       // cos(2*pi*k/11)
  float shh[kParTH];      // sin(2*pi*k/11)
  float thr[kParFreq];    // tau_low + (tau_high - tau_low) * r^p
  float fy[kParTH];       // 2*pi*fftfreq(11)
  float fx[kParWF];       // 2*pi*rfftfreq(10)
};

struct ParParams {
  const __nv_bfloat16 *active;  // [A, HW, C]
  __nv_bfloat16 *full;          // [T, HW, C]
  int C, HW, n_chunks;
  int n_pairs, n_targets;
  int pair_left[kParMaxPairs], pair_right[kParMaxPairs];  // rows of `active`
  int target_pair[kParMaxTargets];                        // index into pairs
  int target_frame[kParMaxTargets];                       // frame row of `full`
  float target_alpha[kParMaxTargets];
  float temperature;
  int ramp_confidence;
  const float *tile_confidence;  // [n_pairs, 18] or null
  float *partials;               // [n_pairs, 18, n_chunks, 198]
  float *weights;                // [n_targets, 18, 66, 4]
  float *pred;                   // [n_targets, 18, 110, C]
  uint8_t *filters;              // [n_targets, 18] F images (hi, lo), kParFilterBytes each
  float *stats;                  // optional, see stats layout in capi
  ParTables tab;
};

__device__ __forceinline__ int reflect_idx(int i, int n) {
  if (i < 0) i = -i;
  if (i >= n) i = 2 * (n - 1) - i;
  return i;
}

// Spectra live in shared memory, one column per thread (channel): entry e of
// a thread's column is col[e * ld].  Layout of a 66-bin spectrum: bin
// f = ky*6+kx at entries 2f (re) and 2f+1 (im); the row-transform stage uses
// the same slots (row i, bin kx) before the column stage overwrites them.

// Windowed reflect-padded tile -> rfft2 (unnormalised, as torch.fft.rfft2).
__device__ __forceinline__ void rfft2_to_smem(const __nv_bfloat16 *frame, int C, int c, int tile,
                                              const ParTables &tab, float *col, int ld) {
  const int gy = tile / kParGW, gx = tile % kParGW;
  int xs[kParTW];
#pragma unroll
  for (int j = 0; j < kParTW; ++j) xs[j] = reflect_idx(gx * kParStride + j - kParPadW, kParW);
#pragma unroll 1
  for (int i = 0; i < kParTH; ++i) {
    const int y = reflect_idx(gy * kParStride + i - kParPadH, kParH);
    float r[kParTW];
#pragma unroll
    for (int j = 0; j < kParTW; ++j)
      r[j] = __bfloat162float(frame[(size_t)(y * kParW + xs[j]) * C + c]) * tab.win[i * kParTW + j];
    float a[5], b[5];
#pragma unroll
    for (int n = 1; n <= 4; ++n) {
      a[n] = r[n] + r[kParTW - n];
      b[n] = r[n] - r[kParTW - n];
    }
#pragma unroll
    for (int k = 0; k < kParWF; ++k) {
      float re = r[0] + ((k & 1) ? -r[5] : r[5]);
      float im = 0.0f;
#pragma unroll
      for (int n = 1; n <= 4; ++n) {
        const int m = (k * n) % kParTW;
        re = fmaf(a[n], tab.cw[m], re);
        im = fmaf(-b[n], tab.sw[m], im);
      }
      col[(2 * (i * kParWF + k)) * ld] = re;
      col[(2 * (i * kParWF + k) + 1) * ld] = im;
    }
  }
#pragma unroll 1
  for (int k = 0; k < kParWF; ++k) {
    float Rr[kParTH], Ri[kParTH];
#pragma unroll
    for (int n = 0; n < kParTH; ++n) {
      Rr[n] = col[(2 * (n * kParWF + k)) * ld];
      Ri[n] = col[(2 * (n * kParWF + k) + 1) * ld];
    }
    float sr[6], si[6], dr[6], di[6];
    float tr = Rr[0], ti = Ri[0];
#pragma unroll
    for (int n = 1; n <= 5; ++n) {
      sr[n] = Rr[n] + Rr[kParTH - n];
      si[n] = Ri[n] + Ri[kParTH - n];
      dr[n] = Rr[n] - Rr[kParTH - n];
      di[n] = Ri[n] - Ri[kParTH - n];
      tr += sr[n];
      ti += si[n];
    }
    col[(2 * k) * ld] = tr;
    col[(2 * k + 1) * ld] = ti;
#pragma unroll
    for (int ky = 1; ky <= 5; ++ky) {
      float ar = Rr[0], ai = Ri[0], br = 0.0f, bi = 0.0f;
#pragma unroll
      for (int n = 1; n <= 5; ++n) {
        const int m = (ky * n) % kParTH;
        ar = fmaf(sr[n], tab.ch[m], ar);
        ai = fmaf(si[n], tab.ch[m], ai);
        br = fmaf(dr[n], tab.shh[m], br);
        bi = fmaf(di[n], tab.shh[m], bi);
      }
      // X[ky] = A - iB, X[11-ky] = A + iB
      col[(2 * (ky * kParWF + k)) * ld] = ar + bi;
      col[(2 * (ky * kParWF + k) + 1) * ld] = ai - br;
      col[(2 * ((kParTH - ky) * kParWF + k)) * ld] = ar - bi;
      col[(2 * ((kParTH - ky) * kParWF + k) + 1) * ld] = ai + br;
    }
  }
}

// In place: spectrum -> inverse along H (Z, unnormalised); then the c2r rows
// (imaginary parts of bins kx = 0 and 5 dropped) give x = irfft2(X, s=(11,10))
// which is multiplied by the synthesis window and stored to out[i*ostride].
__device__ __forceinline__ void irfft2_from_smem(float *col, int ld, const ParTables &tab,
                                                 float *out, size_t ostride, bool store) {
#pragma unroll 1
  for (int k = 0; k < kParWF; ++k) {
    float Xr[kParTH], Xi[kParTH];
#pragma unroll
    for (int n = 0; n < kParTH; ++n) {
      Xr[n] = col[(2 * (n * kParWF + k)) * ld];
      Xi[n] = col[(2 * (n * kParWF + k) + 1) * ld];
    }
    float sr[6], si[6], dr[6], di[6];
    float tr = Xr[0], ti = Xi[0];
#pragma unroll
    for (int n = 1; n <= 5; ++n) {
      sr[n] = Xr[n] + Xr[kParTH - n];
      si[n] = Xi[n] + Xi[kParTH - n];
      dr[n] = Xr[n] - Xr[kParTH - n];
      di[n] = Xi[n] - Xi[kParTH - n];
      tr += sr[n];
      ti += si[n];
    }
    col[(2 * k) * ld] = tr;
    col[(2 * k + 1) * ld] = ti;
#pragma unroll
    for (int y = 1; y <= 5; ++y) {
      float ar = Xr[0], ai = Xi[0], br = 0.0f, bi = 0.0f;
#pragma unroll
      for (int n = 1; n <= 5; ++n) {
        const int m = (y * n) % kParTH;
        ar = fmaf(sr[n], tab.ch[m], ar);
        ai = fmaf(si[n], tab.ch[m], ai);
        br = fmaf(dr[n], tab.shh[m], br);
        bi = fmaf(di[n], tab.shh[m], bi);
      }
      // Z[y] = A + iB, Z[11-y] = A - iB
      col[(2 * (y * kParWF + k)) * ld] = ar - bi;
      col[(2 * (y * kParWF + k) + 1) * ld] = ai + br;
      col[(2 * ((kParTH - y) * kParWF + k)) * ld] = ar + bi;
      col[(2 * ((kParTH - y) * kParWF + k) + 1) * ld] = ai - br;
    }
  }
  const float norm = 1.0f / (float)(kParTH * kParTW);
#pragma unroll 1
  for (int y = 0; y < kParTH; ++y) {
    float zr[kParWF], zi[kParWF];
#pragma unroll
    for (int k = 0; k < kParWF; ++k) {
      zr[k] = col[(2 * (y * kParWF + k)) * ld];
      zi[k] = col[(2 * (y * kParWF + k) + 1) * ld];
    }
    float e[6], o[6];
#pragma unroll
    for (int xx = 0; xx <= 5; ++xx) {
      float cc = zr[0] + ((xx & 1) ? -zr[5] : zr[5]), ss = 0.0f;
#pragma unroll
      for (int k = 1; k <= 4; ++k) {
        const int m = (k * xx) % kParTW;
        cc = fmaf(2.0f * zr[k], tab.cw[m], cc);
        ss = fmaf(2.0f * zi[k], tab.sw[m], ss);
      }
      e[xx] = cc;
      o[xx] = ss;
    }
    if (store) {
      float v[kParTW];
      v[0] = e[0];
      v[5] = e[5];
#pragma unroll
      for (int xx = 1; xx <= 4; ++xx) {
        v[xx] = e[xx] - o[xx];
        v[kParTW - xx] = e[xx] + o[xx];
      }
#pragma unroll
      for (int xx = 0; xx < kParTW; ++xx)
        out[(size_t)(y * kParTW + xx) * ostride] = v[xx] * norm * tab.win[y * kParTW + xx];
    }
  }
}

// ---------------------------------------------------------------------------
// grid (chunk, tile, pair), kParChunk threads.  Dynamic smem: two spectra.
__global__ void __launch_bounds__(kParChunk) par_stats_kernel(const ParParams p) {
  extern __shared__ float psm[];
  constexpr int ld = kParChunk + 1;
  float *sL = psm;                        // [132][ld]
  float *sR = psm + 2 * kParFreq * ld;    // [132][ld]
  const int chunk = blockIdx.x, tile = blockIdx.y, pair = blockIdx.z;
  const int c = chunk * kParChunk + threadIdx.x;
  const bool valid = c < p.C;
  const int cc = valid ? c : 0;
  float *colL = sL + threadIdx.x, *colR = sR + threadIdx.x;
  rfft2_to_smem(p.active + (size_t)p.pair_left[pair] * p.HW * p.C, p.C, cc, tile, p.tab, colL, ld);
  rfft2_to_smem(p.active + (size_t)p.pair_right[pair] * p.HW * p.C, p.C, cc, tile, p.tab, colR, ld);
  // R * conj(L) per bin: re -> sL[f], im -> sL[66+f], |.| -> sL[132+f]
  // (sL rows 66..131 are L's own values, read before they are overwritten
  // because bin f reads rows 2f, 2f+1 of L and writes rows f, 66+f, 132+f
  // only after every bin with a larger row index has been read: the values
  // are first gathered into registers per bin range.)
  float cre[kParFreq], cim[kParFreq];
#pragma unroll
  for (int f = 0; f < kParFreq; ++f) {
    const float lr = colL[(2 * f) * ld], li = colL[(2 * f + 1) * ld];
    const float rr = colR[(2 * f) * ld], ri = colR[(2 * f + 1) * ld];
    cre[f] = valid ? rr * lr + ri * li : 0.0f;
    cim[f] = valid ? ri * lr - rr * li : 0.0f;
  }
#pragma unroll
  for (int f = 0; f < kParFreq; ++f) {
    colL[f * ld] = cre[f];
    colL[(kParFreq + f) * ld] = cim[f];
    colR[f * ld] = sqrtf(cre[f] * cre[f] + cim[f] * cim[f]);
  }
  __syncthreads();
  float *dst = p.partials + (((size_t)pair * kParTiles + tile) * p.n_chunks + chunk) * kParPartial;
  for (int r = threadIdx.x; r < kParPartial; r += blockDim.x) {
    const float *row = r < 2 * kParFreq ? sL + (size_t)r * ld : sR + (size_t)(r - 2 * kParFreq) * ld;
    float acc = 0.0f;
    for (int j = 0; j < kParChunk; ++j) acc += row[j];
    dst[r] = acc;
  }
}

// ---------------------------------------------------------------------------
// One CTA per (tile, pair), 128 threads.
__global__ void __launch_bounds__(128) par_finalize_kernel(const ParParams p) {
  __shared__ float part[kParPartial];
  __shared__ float unit_re[kParFreq], unit_im[kParFreq], coh[kParFreq], wgt[kParFreq];
  __shared__ float theta[kParFreq], corr[kParPix];
  __shared__ float s_base, s_denom, s_conf, s_dx, s_dy, s_ramp;
  const int tile = blockIdx.x, pair = blockIdx.y, t = threadIdx.x;
  const float *src = p.partials + ((size_t)pair * kParTiles + tile) * p.n_chunks * kParPartial;
  for (int r = t; r < kParPartial; r += blockDim.x) {
    float acc = 0.0f;
    for (int ch = 0; ch < p.n_chunks; ++ch) acc += src[(size_t)ch * kParPartial + r];
    part[r] = acc;
  }
  __syncthreads();
  if (t < kParFreq) {
    const float sr = part[t], si = part[kParFreq + t], energy = part[2 * kParFreq + t];
    const float mag = sqrtf(sr * sr + si * si);
    const float co = mag / fmaxf(energy, 1e-8f);
    coh[t] = co;
    wgt[t] = t == 0 ? 0.0f : energy;
    float ur = 1.0f, ui = 0.0f;
    if (mag > 1e-8f) {
      const float m = fmaxf(mag, 1e-8f);
      ur = sr / m;
      ui = si / m;
    }
    unit_re[t] = ur;
    unit_im[t] = ui;
    theta[t] = t == 0 ? 0.0f : atan2f(ui, ur);
  }
  __syncthreads();
  // Weighted sums over the 66 frequencies (warp 0; fixed shuffle tree).
  if (t < 32) {
    float w = 0.0f, cw = 0.0f;
    for (int f = t; f < kParFreq; f += 32) {
      w += wgt[f];
      cw += coh[f] * wgt[f];
    }
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) {
      w += __shfl_xor_sync(0xffffffffu, w, s);
      cw += __shfl_xor_sync(0xffffffffu, cw, s);
    }
    if (t == 0) {
      const float denom = fmaxf(w, 1e-8f);
      s_denom = denom;
      s_base = fminf(fmaxf(cw / denom, 0.0f), 1.0f);
    }
  }
  // PHAT correlation: irfft2(unit * coherence, s=(11,10)), one output per thread.
  if (t < kParPix) {
    const int y = t / kParTW, x = t % kParTW;
    float acc = 0.0f;
    for (int ky = 0; ky < kParTH; ++ky) {
      const int my = (ky * y) % kParTH;
      const float ey_c = p.tab.ch[my], ey_s = p.tab.shh[my];
      for (int kx = 0; kx < kParWF; ++kx) {
        const int f = ky * kParWF + kx;
        const float vr = unit_re[f] * coh[f], vi = unit_im[f] * coh[f];
        // Z contribution: v * e^{+i 2pi ky y/11}
        const float zr = vr * ey_c - vi * ey_s, zi = vr * ey_s + vi * ey_c;
        if (kx == 0) {
          acc += zr;
        } else if (kx == 5) {
          acc += (x & 1) ? -zr : zr;
        } else {
          const int mx = (kx * x) % kParTW;
          acc += 2.0f * (zr * p.tab.cw[mx] - zi * p.tab.sw[mx]);
        }
      }
    }
    corr[t] = acc * (1.0f / (float)(kParTH * kParTW));
  }
  __syncthreads();
  if (t == 0) {
    int best = 0;
    float bv = corr[0];
    for (int i = 1; i < kParPix; ++i)
      if (corr[i] > bv) {
        bv = corr[i];
        best = i;
      }
    const int py = best / kParTW, px = best % kParTW;
    auto sub = [](float before, float middle, float after) {
      const float den = before - 2.0f * middle + after;
      return fabsf(den) > 1e-8f ? fminf(fmaxf(0.5f * (before - after) / den, -0.5f), 0.5f) : 0.0f;
    };
    const float xl = corr[py * kParTW + (px + kParTW - 1) % kParTW];
    const float xr = corr[py * kParTW + (px + 1) % kParTW];
    const float yu = corr[((py + kParTH - 1) % kParTH) * kParTW + px];
    const float yd = corr[((py + 1) % kParTH) * kParTW + px];
    s_dx = (float)(px >= (kParTW + 1) / 2 ? px - kParTW : px) + sub(xl, bv, xr);
    s_dy = (float)(py >= (kParTH + 1) / 2 ? py - kParTH : py) + sub(yu, bv, yd);
  }
  __syncthreads();
  if (t < 32) {
    float acc = 0.0f;
    for (int f = t; f < kParFreq; f += 32) {
      const int ky = f / kParWF, kx = f % kParWF;
      const float ang = -(s_dy * p.tab.fy[ky] + s_dx * p.tab.fx[kx]);
      float sa, ca;
      sincosf(ang, &sa, &ca);
      // Re(unit * conj(exp(i ang)))
      const float circ = fminf(fmaxf(unit_re[f] * ca + unit_im[f] * sa, 0.0f), 1.0f);
      acc += circ * wgt[f];
    }
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, s);
    if (t == 0) {
      s_ramp = fminf(fmaxf(acc / s_denom, 0.0f), 1.0f);
      float conf = s_base;
      if (p.ramp_confidence) conf = conf * s_ramp;
      conf = fminf(fmaxf(conf, 0.0f), 1.0f);
      if (p.tile_confidence) conf = p.tile_confidence[pair * kParTiles + tile];
      s_conf = conf;
    }
  }
  __syncthreads();
  if (t < kParFreq) {
    const float z = (s_conf - p.tab.thr[t]) / p.temperature;
    const float g = 1.0f / (1.0f + expf(-z));
    for (int tg = 0; tg < p.n_targets; ++tg) {
      if (p.target_pair[tg] != pair) continue;
      const float a = p.target_alpha[tg];
      float sl, cl, sr, cr;
      sincosf((g * a) * theta[t], &sl, &cl);
      sincosf((-g * (1.0f - a)) * theta[t], &sr, &cr);
      float *w = p.weights + (((size_t)tg * kParTiles + tile) * kParFreq + t) * 4;
      w[0] = (1.0f - a) * cl;
      w[1] = (1.0f - a) * sl;
      w[2] = a * cr;
      w[3] = a * sr;
    }
    if (p.stats) {
      // per pair: theta[18*66], conf[18], g[18*66], disp[18*2], base[18], ramp[18]
      float *st = p.stats + (size_t)pair * (kParTiles * (2 * kParFreq + 5));
      st[tile * kParFreq + t] = theta[t];
      st[kParTiles * (kParFreq + 1) + tile * kParFreq + t] = g;
      if (t == 0) {
        st[kParTiles * kParFreq + tile] = s_conf;
        st[kParTiles * (2 * kParFreq + 1) + 2 * tile] = s_dx;
        st[kParTiles * (2 * kParFreq + 1) + 2 * tile + 1] = s_dy;
        st[kParTiles * (2 * kParFreq + 3) + tile] = s_base;
        st[kParTiles * (2 * kParFreq + 4) + tile] = s_ramp;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// grid (chunk, tile, pair), kParChunk threads.  Dynamic smem: three spectra.
__global__ void __launch_bounds__(kParChunk) par_predict_kernel(const ParParams p) {
  extern __shared__ float psm[];
  constexpr int ld = kParChunk + 1;
  float *sL = psm, *sR = psm + 2 * kParFreq * ld, *sZ = psm + 4 * kParFreq * ld;
  __shared__ float w_s[kParFreq * 4];
  const int chunk = blockIdx.x, tile = blockIdx.y, pair = blockIdx.z;
  const int c = chunk * kParChunk + threadIdx.x;
  const bool valid = c < p.C;
  const int cc = valid ? c : 0;
  float *colL = sL + threadIdx.x, *colR = sR + threadIdx.x, *colZ = sZ + threadIdx.x;
  rfft2_to_smem(p.active + (size_t)p.pair_left[pair] * p.HW * p.C, p.C, cc, tile, p.tab, colL, ld);
  rfft2_to_smem(p.active + (size_t)p.pair_right[pair] * p.HW * p.C, p.C, cc, tile, p.tab, colR, ld);
  for (int tg = 0; tg < p.n_targets; ++tg) {
    if (p.target_pair[tg] != pair) continue;
    __syncthreads();
    for (int i = threadIdx.x; i < kParFreq * 4; i += blockDim.x)
      w_s[i] = p.weights[((size_t)tg * kParTiles + tile) * kParFreq * 4 + i];
    __syncthreads();
#pragma unroll 6
    for (int f = 0; f < kParFreq; ++f) {
      const float lr = colL[(2 * f) * ld], li = colL[(2 * f + 1) * ld];
      const float rr = colR[(2 * f) * ld], ri = colR[(2 * f + 1) * ld];
      const float wlr = w_s[4 * f], wli = w_s[4 * f + 1], wrr = w_s[4 * f + 2], wri = w_s[4 * f + 3];
      // mixed = L*wl + R*wr
      colZ[(2 * f) * ld] = (lr * wlr - li * wli) + (rr * wrr - ri * wri);
      colZ[(2 * f + 1) * ld] = (lr * wli + li * wlr) + (rr * wri + ri * wrr);
    }
    float *dst = p.pred + ((size_t)tg * kParTiles + tile) * kParPix * p.C + cc;
    irfft2_from_smem(colZ, ld, p.tab, dst, (size_t)p.C, valid);
  }
}

// ---------------------------------------------------------------------------
// Tensor-core prediction.
constexpr int kParMmaTargets = 4;                // targets per pair (TMEM: 4 x 112 columns)
constexpr int kParK = 224;                       // L pixels 0..109, R pixels 112..221
constexpr int kParN = 112;                       // output pixels (110 used)
constexpr int kParKChunks = 4;                   // 64-element K chunks of the F image
constexpr int kParFChunkBytes = kParN * 128;     // 14336
constexpr int kParFHalfBytes = kParKChunks * kParFChunkBytes;  // hi or lo: 57344
constexpr int kParFilterBytes = 2 * kParFHalfBytes;            // 114688
constexpr int kParAHalfBytes = kParK * 128;      // 64 channels x 224 rows: 28672

struct ParMmaSmem {
  static constexpr int a = 0;                          // 2 x kParAHalfBytes
  static constexpr int b = 2 * kParAHalfBytes;         // kParFilterBytes
  static constexpr int bars = b + kParFilterBytes;     // a_full, b_full, mma_done[4]
  static constexpr int tmem_slot = bars + (2 + kParMmaTargets) * 8;
  static constexpr int total = tmem_slot + 16;
  static constexpr int alloc = total + 1024;
};

// grid (tile, target, K chunk), 256 threads.
__global__ void __launch_bounds__(256) par_filter_kernel(const ParParams p) {
  __shared__ float wl_re[kParFreq], wl_im[kParFreq], wr_re[kParFreq], wr_im[kParFreq];
  __shared__ float kern[2][kParPix];
  const int tile = blockIdx.x, tg = blockIdx.y, t = threadIdx.x;
  const float *w = p.weights + ((size_t)tg * kParTiles + tile) * kParFreq * 4;
  if (t < kParFreq) {
    wl_re[t] = w[4 * t];
    wl_im[t] = w[4 * t + 1];
    wr_re[t] = w[4 * t + 2];
    wr_im[t] = w[4 * t + 3];
  }
  __syncthreads();
  if (t < 2 * kParPix) {
    const int side = t / kParPix, d = t % kParPix;
    const int dy = d / kParTW, dx = d % kParTW;
    const float *are = side ? wr_re : wl_re, *aim = side ? wr_im : wl_im;
    float acc = 0.0f;
    for (int ky = 0; ky < kParTH; ++ky) {
      const int my = (ky * dy) % kParTH;
      const float cy = p.tab.ch[my], sy = p.tab.shh[my];
      for (int kx = 0; kx < kParWF; ++kx) {
        const int mx = (kx * dx) % kParTW;
        const float cx = p.tab.cw[mx], sx = p.tab.sw[mx];
        // e^{i(2pi ky dy/11 + 2pi kx dx/10)}
        const float er = cy * cx - sy * sx, ei = sy * cx + cy * sx;
        const int f = ky * kParWF + kx;
        const float re = are[f] * er - aim[f] * ei;
        acc += (kx == 0 || kx == kParWF - 1) ? re : 2.0f * re;
      }
    }
    kern[side][d] = acc * (1.0f / (float)kParPix);
  }
  __syncthreads();
  // F image: element (n, k) at chunk k/64, row n, 16-byte group (k%64)/8
  // swizzled by n & 7 (128-byte swizzle, K-major).
  uint8_t *img = p.filters + ((size_t)tg * kParTiles + tile) * kParFilterBytes;
  const int kc0 = blockIdx.z;  // this CTA's 64-element K chunk
  const int g_end = min(8, kParK / 8 - kc0 * 8);
  for (int e = t; e < kParN * g_end; e += blockDim.x) {
    const int n = e / g_end, g = kc0 * 8 + e % g_end;  // 8 consecutive k
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      float v[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int k = g * 8 + j + u;
        float f = 0.0f;
        const int side = k < kParN ? 0 : 1;
        const int q = k - side * kParN;
        if (n < kParPix && q < kParPix) {
          const int dy = (n / kParTW - q / kParTW + kParTH) % kParTH;
          const int dx = (n % kParTW - q % kParTW + kParTW) % kParTW;
          f = p.tab.win[n] * p.tab.win[q] * kern[side][dy * kParTW + dx];
        }
        v[u] = f;
      }
      const __nv_bfloat162 h = __floats2bfloat162_rn(v[0], v[1]);
      const float2 hf = __bfloat1622float2(h);
      const __nv_bfloat162 l = __floats2bfloat162_rn(v[0] - hf.x, v[1] - hf.y);
      hi[j / 2] = *reinterpret_cast<const uint32_t *>(&h);
      lo[j / 2] = *reinterpret_cast<const uint32_t *>(&l);
    }
    const int kc = g / 8, grp = g % 8;
    const size_t off = (size_t)kc * kParFChunkBytes + (size_t)n * 128 + ((grp ^ (n & 7)) * 16);
    *reinterpret_cast<uint4 *>(img + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4 *>(img + kParFHalfBytes + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  }
}

// grid (chunk of 128 channels, tile, pair), 128 threads.
__global__ void __launch_bounds__(128, 1)
    par_predict_mma_kernel(const ParParams p) {
  extern __shared__ uint8_t par_smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(par_smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + ParMmaSmem::bars);
  uint64_t *b_full = bars + 1;
  uint64_t *mma_done = bars + 2;  // one per target of the pair: each completes once
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + ParMmaSmem::tmem_slot);
  int *err = &g_cast_device_error;
  const int chunk = blockIdx.x, tile = blockIdx.y, pair = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gy = tile / kParGW, gx = tile % kParGW;

  if (threadIdx.x == 0) {
    castdev::mbar_init(b_full, 1);
    for (int i = 0; i < kParMmaTargets; ++i) castdev::mbar_init(&mma_done[i], 1);
    castdev::fence_barrier_init();
  }
  if (warp == 0) {
    castdev::tmem_alloc(tmem_slot, 512);
    castdev::tmem_relinquish();
  }
  // zero K padding rows 110, 111, 222, 223 of both channel halves
  if (threadIdx.x < 2 * 4 * 8) {
    const int h = threadIdx.x / 32, r = (threadIdx.x / 8) % 4, c16 = threadIdx.x % 8;
    const int row = r < 2 ? kParPix + r : kParN + kParPix + (r - 2);
    *reinterpret_cast<uint4 *>(smem + ParMmaSmem::a + h * kParAHalfBytes + row * 128 + c16 * 16) =
        make_uint4(0u, 0u, 0u, 0u);
  }

  // A: 2 anchors x 110 pixels x 128 channels, 16-byte cp.async copies by all
  // threads into the 128-byte-swizzled MN-major layout (channels beyond C
  // are zero-filled); the reflect padding is in the source row.
  {
    const uint32_t a_s = castdev::smem_u32(smem + ParMmaSmem::a);
    for (int e = threadIdx.x; e < 2 * kParPix * 16; e += blockDim.x) {
      const int g16 = e % 16, pix = e / 16;  // 16 groups of 8 channels per pixel
      const int side = pix / kParPix, q = pix % kParPix;
      const int frame_row = side ? p.pair_right[pair] : p.pair_left[pair];
      const int y = reflect_idx(gy * kParStride + q / kParTW - kParPadH, kParH);
      const int x = reflect_idx(gx * kParStride + q % kParTW - kParPadW, kParW);
      const int krow = side * kParN + q, h = g16 / 8, g = g16 % 8;
      const int c0 = chunk * 128 + g16 * 8;
      const uint32_t dst = a_s + h * kParAHalfBytes + krow * 128 + ((g ^ (krow & 7)) * 16);
      const __nv_bfloat16 *src = p.active + ((size_t)frame_row * p.HW + y * kParW + x) * p.C + c0;
      const uint32_t bytes = c0 < p.C ? 16u : 0u;  // zero-fill past C
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst),
                   "l"(c0 < p.C ? src : p.active), "r"(bytes)
                   : "memory");
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
  }

  // the cp.async writes and the zero rows are generic-proxy writes the MMAs
  // (async proxy) read
  castdev::fence_proxy_async_smem();
  __syncthreads();
  castdev::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const uint32_t sbase = castdev::smem_u32(smem);
  constexpr uint32_t idesc = castdev::make_idesc(1, 1, 1, 1, 0, 128, kParN);
  int local = 0;  // this target's index among the pair's targets (TMEM columns)
  int b_loads = 0;
  bool ok = true;
  for (int tg = 0; tg < p.n_targets; ++tg) {
    if (p.target_pair[tg] != pair) continue;
    const uint32_t d_col = tmem + local * kParN;
    if (threadIdx.x == 0 && ok) {
      // the previous target's MMAs have finished reading B
      if (local > 0) ok = castdev::mbar_wait(&mma_done[local - 1], 0, err);
      if (ok) {
        castdev::mbar_arrive_expect_tx(b_full, kParFilterBytes);
        castdev::bulk_load(smem + ParMmaSmem::b,
                           p.filters + ((size_t)tg * kParTiles + tile) * kParFilterBytes,
                           kParFilterBytes, b_full);
        ++b_loads;
      }
      if (ok) ok = castdev::mbar_wait(b_full, local & 1, err);
      if (ok) {
        castdev::tc_fence_after();
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {  // F hi, then F lo
#pragma unroll
          for (int s = 0; s < kParK / 16; ++s) {
            const uint64_t ad = castdev::smem_desc_sw128(sbase + ParMmaSmem::a + 2048 * s,
                                                         kParAHalfBytes, 1024);
            const uint64_t bd = castdev::smem_desc_sw128(
                sbase + ParMmaSmem::b + half * kParFHalfBytes + (s >> 2) * kParFChunkBytes +
                    (s & 3) * 32,
                16, 1024);
            castdev::mma_f16_ss(d_col, ad, bd, idesc, (half | s) != 0);
          }
        }
        castdev::tc_commit(&mma_done[local]);
      }
    }
    // epilogue: this target's 110 predicted pixels for the warp's 32 channels
    const bool done = __all_sync(0xffffffffu, castdev::mbar_wait(&mma_done[local], 0, err));
    castdev::tc_fence_after();
    const int c = chunk * 128 + warp * 32 + lane;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    float *dst = p.pred + ((size_t)tg * kParTiles + tile) * kParPix * p.C + c;
#pragma unroll 1
    for (int cc = 0; cc < 4; ++cc) {
      uint32_t v[32];
      if (cc < 3) {
        castdev::tmem_ld32(tmem + lane_off + local * kParN + 32 * cc, v);
      } else {
        castdev::tmem_ld16(tmem + lane_off + local * kParN + 96, *reinterpret_cast<uint32_t(*)[16]>(v));
      }
      castdev::tmem_wait_ld();
      const int n_cols = cc < 3 ? 32 : kParPix - 96;
      if (done && c < p.C) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < n_cols) dst[(size_t)(32 * cc + j) * p.C] = __uint_as_float(v[j]);
      }
    }
    ++local;
  }
  // every TMA copy and MMA of this CTA has completed before TMEM is released
  if (threadIdx.x == 0 && b_loads > 0) castdev::mbar_wait_drain(b_full, (b_loads - 1) & 1, err);
  __syncthreads();
  if (warp == 0) {
    castdev::tc_fence_after();
    castdev::tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// grid (HW, n_targets); each thread handles 4 channels.
__global__ void __launch_bounds__(256) par_ola_kernel(const ParParams p) {
  const int pix = blockIdx.x, tg = blockIdx.y;
  const int y = pix / kParW, x = pix % kParW;
  int tiles[4], offs[4], n = 0;
  float norm = 0.0f;
  for (int gy = 0; gy < kParGH; ++gy) {
    const int ty = y + kParPadH - gy * kParStride;
    if (ty < 0 || ty >= kParTH) continue;
    for (int gx = 0; gx < kParGW; ++gx) {
      const int tx = x + kParPadW - gx * kParStride;
      if (tx < 0 || tx >= kParTW) continue;
      const float w = p.tab.win[ty * kParTW + tx];
      norm += w * w;
      tiles[n] = gy * kParGW + gx;
      offs[n] = ty * kParTW + tx;
      ++n;
    }
  }
  const float inv = 1.0f / norm;
  __nv_bfloat16 *dst = p.full + ((size_t)p.target_frame[tg] * p.HW + pix) * p.C;
  for (int c4 = threadIdx.x * 4; c4 < p.C; c4 += blockDim.x * 4) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i = 0; i < n; ++i) {
      const float4 v = *reinterpret_cast<const float4 *>(
          p.pred + (((size_t)tg * kParTiles + tiles[i]) * kParPix + offs[i]) * p.C + c4);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x * inv, acc.y * inv);
    __nv_bfloat162 hi = __floats2bfloat162_rn(acc.z * inv, acc.w * inv);
    uint2 packed;
    packed.x = *reinterpret_cast<uint32_t *>(&lo);
    packed.y = *reinterpret_cast<uint32_t *>(&hi);
    *reinterpret_cast<uint2 *>(dst + c4) = packed;
  }
}

}  // namespace castk
