// Phase-Aware Reconstruction (FC-PASM reference numerics) for sm_100a.
//
// Restates proposed/matrix_world_spectral_residual.py:2771-3662 with the
// factory knobs.  Per-channel path (any C): the 11x10 tile transforms are
// small direct real DFTs in registers (one thread per channel).
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
// Tensor-core paths (used when C % 8 == 0 and the anchors are 16-byte
// aligned; the prediction also needs at most kParMmaTargets targets per
// pair).  The statistics' rfft2 is a fixed linear map of a tile's pixels,
// and the whole prediction chain analysis window -> rfft2 -> per-frequency
// mix -> irfft2 -> synthesis window is linear in the two anchor tiles and
// circular in the pixel offset: a target's predicted tile is
// pred = F_L l + F_R r with F[p][q] = win[p] win[q] kern[(p - q) mod (11, 10)]
// and kern[d] = (1/110) sum_f c_kx Re(w_f e^{i w_f . d}) (c_kx = 1 for
// kx = 0, 5, else 2: the c2r rows).  Both become GEMMs with the channels as M.
//   par_stats_mma_kernel persistent, CTAs per tile class: the class's
//                        windowed rfft2 matrix (110 independent real
//                        columns, reflect slots folded in) built in shared
//                        memory as a bf16 hi + lo image, anchor tiles by TMA
//                        into two buffers, spectra by tcgen05.mma into two
//                        TMEM halves, R conj(L) and |R conj(L)| summed over a
//                        chunk's channels by warp butterflies -> partials
//   par_finalize_kernel  as above
//   par_filter_kernel    grid (tile, target, K chunk): kern for L and R from
//                        the mix weights, then F as bf16 hi + lo (the pair
//                        carries ~16 significant bits) in the shared-memory
//                        image the MMA reads, in the slot order of the
//                        prediction's TMA boxes
//   par_predict_mma_kernel persistent over (target, tile, 128-channel
//                        chunk): one TMA box per anchor and channel half,
//                        D[128 ch x 112 px] = A[128 ch x 224 (L|R slots)] F
//                        via tcgen05.mma (A MN-major, F K-major, fp32 in
//                        TMEM), then the predicted tiles to the workspace
//   par_ola_kernel       as above
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
  int n_stat_chunks;            // chunks of `partials` (64 or 128 channels each)
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
  int stat_cta_start[10];        // tensor-core statistics: first CTA of each tile class (9 = grid)
  uint8_t *dft;                  // per tile class: windowed rfft2 matrix image (hi, lo), kParDftBytes each
  float *stats;                  // optional, see stats layout in capi
  ParTables tab;
};


__device__ __forceinline__ int reflect_idx(int i, int n) {
  if (i < 0) i = -i;
  if (i >= n) i = 2 * (n - 1) - i;
  return i;
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

// Prediction: two A buffers (2 x kParAHalfBytes each), one F image, then
// a_full[2], b_full, mma_done[2], tmem_free[2] and the TMEM slot.
struct ParMmaSmem {
  static constexpr int a = 0;
  static constexpr int b = 4 * kParAHalfBytes;
  static constexpr int bars = b + kParFilterBytes;
  static constexpr int tmem_slot = bars + 7 * 8;
  static constexpr int total = tmem_slot + 8;
  static constexpr int alloc = total + 1024;
};
static_assert(ParMmaSmem::alloc <= 227 * 1024, "prediction shared memory");
constexpr int kParEpiWarps = 8;                          // 2 per TMEM lane quarter
constexpr int kParPredThreads = (kParEpiWarps + 1) * 32;  // + the producer / MMA warp
constexpr int kParGatherBytes = 2 * 2 * kParPix * 128;     // both anchors, both channel halves

// The tensor-core paths load a tile as one TMA box of 11 frame rows x 10
// frame columns, clamped into the frame: every reflected pixel the tile
// needs lies inside it.  Tile pixel (i, j) sits in box slot (r, s) =
// (reflect(y) - y0, reflect(x) - x0); at the frame edges two tile pixels can
// share a slot and some slots are unused, which the F and Dft images absorb
// (coefficients of pixels sharing a slot are summed, unused slots are zero).
__host__ __device__ __forceinline__ int par_box_y0(int gy) {
  const int y = gy * kParStride - kParPadH;
  return y < 0 ? 0 : (y > kParH - kParTH ? kParH - kParTH : y);
}
__host__ __device__ __forceinline__ int par_box_x0(int gx) {
  const int x = gx * kParStride - kParPadW;
  return x < 0 ? 0 : (x > kParW - kParTW ? kParW - kParTW : x);
}

// Tile rows (bits 0-7, 4 each) and tile columns (bits 8-15) whose pixels sit
// in box slot `slot` of tile (gy, gx), with their counts in bits 16-17 and
// 20-21: at most two of each.
__device__ __forceinline__ uint32_t par_slot_word(int gy, int gx, int slot) {
  const int r = slot / kParTW, sx = slot % kParTW;
  uint32_t rows = 0, cols = 0, packed = 0;
  for (int i = 0; i < kParTH; ++i)
    if (reflect_idx(gy * kParStride + i - kParPadH, kParH) - par_box_y0(gy) == r && rows < 2)
      packed |= (uint32_t)i << (4 * rows++);
  for (int j = 0; j < kParTW; ++j)
    if (reflect_idx(gx * kParStride + j - kParPadW, kParW) - par_box_x0(gx) == sx && cols < 2)
      packed |= (uint32_t)j << (8 + 4 * cols++);
  return packed | rows << 16 | cols << 20;
}

// Tile classes: the slot mapping depends only on the tile row gy and on
// whether the tile column is the first, an inner one or the last.
// class = 3 gy + (gx == 0 ? 0 : gx == 5 ? 2 : 1); classes 3 gy + 1 hold 4
// tiles, the others 1.
__host__ __device__ __forceinline__ int par_class_tiles(int cls) { return cls % 3 == 1 ? kParGW - 2 : 1; }
__host__ __device__ __forceinline__ int par_class_tile(int cls, int i) {
  const int gy = cls / 3, c = cls % 3;
  return gy * kParGW + (c == 0 ? 0 : (c == 2 ? kParGW - 1 : 1 + i));
}

// Kernel parameters live in the constant bank, which serves a warp one
// distinct address at a time; kernels that index the tables per lane read a
// shared-memory copy, made here with warp-uniform parameter reads.
__device__ __forceinline__ void par_tables_to_smem(const ParTables &src, ParTables &dst) {
  constexpr int n = (int)(sizeof(ParTables) / 4);
  const float *sp = reinterpret_cast<const float *>(&src);
  float *dp = reinterpret_cast<float *>(&dst);
  const int lane = threadIdx.x & 31;
  for (int base = (threadIdx.x >> 5) * 32; base < n; base += blockDim.x) {
    float mine = 0.0f;
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      if (base + k < n) {
        const float v = sp[base + k];
        mine = lane == k ? v : mine;
      }
    }
    if (base + lane < n) dp[base + lane] = mine;
  }
  __syncthreads();
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

// K chunks kc0 .. kc1-1 of the F image of target tg at `tile`, from its mix
// weights (all threads of the block): kern for L and R, then F as bf16 hi +
// lo (the pair carries ~16 significant bits) in the shared-memory image the
// MMA reads.
struct ParFilterSmem {
  float w[kParFreq][4];                   // wl_re, wl_im, wr_re, wr_im per bin
  float zr[2][kParTH][kParTW], zi[2][kParTH][kParTW];
  float kern[2][kParPix];
  uint32_t slot[kParPix];  // tile pixels in box slot: i0 | i1 << 4 | j0 << 8 | j1 << 12 | rows << 16 | cols << 20
};
__device__ __forceinline__ void par_build_filter(const ParParams &p, const ParTables &tab, int tile, int tg,
                                                 int kc0, int kc1, ParFilterSmem &fs) {
  const int t = threadIdx.x;
  const float *w = p.weights + ((size_t)tg * kParTiles + tile) * kParFreq * 4;
  __syncthreads();  // the previous target's reads of fs are done
  for (int e = t; e < kParFreq * 4; e += blockDim.x) fs.w[e / 4][e % 4] = w[e];
  if (t < kParPix) fs.slot[t] = par_slot_word(tile / kParGW, tile % kParGW, t);
  __syncthreads();
  // kern[d] = (1/110) sum_f c_kx Re(w_f e^{i(2 pi ky dy / 11 + 2 pi kx dx / 10)}),
  // c_kx = 1 for kx = 0, 5 and 2 otherwise: first over kx per (ky, dx) ...
  if (t < 2 * kParPix) {
    const int side = t / kParPix, ky = (t % kParPix) / kParTW, dx = t % kParTW;
    float zr = 0.0f, zi = 0.0f;
#pragma unroll
    for (int kx = 0; kx < kParWF; ++kx) {
      const int m = (kx * dx) % kParTW;
      const float c = (kx == 0 || kx == kParWF - 1) ? 1.0f : 2.0f;
      const float wr = c * fs.w[ky * kParWF + kx][2 * side], wi = c * fs.w[ky * kParWF + kx][2 * side + 1];
      zr += wr * tab.cw[m] - wi * tab.sw[m];
      zi += wr * tab.sw[m] + wi * tab.cw[m];
    }
    fs.zr[side][ky][dx] = zr;
    fs.zi[side][ky][dx] = zi;
  }
  __syncthreads();
  // ... then over ky per (dy, dx)
  if (t < 2 * kParPix) {
    const int side = t / kParPix, dy = (t % kParPix) / kParTW, dx = t % kParTW;
    float acc = 0.0f;
#pragma unroll
    for (int ky = 0; ky < kParTH; ++ky) {
      const int m = (ky * dy) % kParTH;
      acc += fs.zr[side][ky][dx] * tab.ch[m] - fs.zi[side][ky][dx] * tab.shh[m];
    }
    fs.kern[side][t % kParPix] = acc * (1.0f / (float)kParPix);
  }
  __syncthreads();
// F image: element (n, k) at chunk k/64, row n, 16-byte group (k%64)/8
  // swizzled by n & 7 (128-byte swizzle, K-major).
  uint8_t *img = p.filters + ((size_t)tg * kParTiles + tile) * kParFilterBytes;
  const int g0 = kc0 * 8, ng = min(kc1 * 8, kParK / 8) - g0;
  // a warp takes consecutive output pixels n of one group of 8 K slots: the
  // slot words and windows are broadcasts, the kern reads consecutive
  for (int e = t; e < kParN * ng; e += blockDim.x) {
    const int n = e % kParN, g = g0 + e / kParN;  // 8 consecutive k
    const int ny = n / kParTW, nx = n % kParTW;
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      float v[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int k = g * 8 + j + u;
        float f = 0.0f;
        const int side = k < kParN ? 0 : 1;
        const int slot = k - side * kParN;  // box slot r * 10 + s
        if (n < kParPix && slot < kParPix) {
          // sum over the (at most 2 x 2) tile pixels in this slot
          const uint32_t sm = fs.slot[slot];
          const int rows = (sm >> 16) & 3, cols = (sm >> 20) & 3;
#pragma unroll
          for (int a = 0; a < 2; ++a) {
            const int i = (sm >> (4 * a)) & 15;
            int dy = ny - i;
            dy += dy < 0 ? kParTH : 0;
#pragma unroll
            for (int b = 0; b < 2; ++b) {
              const int j = (sm >> (8 + 4 * b)) & 15;
              int dx = nx - j;
              dx += dx < 0 ? kParTW : 0;
              if (a < rows && b < cols) f += tab.win[i * kParTW + j] * fs.kern[side][dy * kParTW + dx];
            }
          }
          f *= tab.win[n];
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

// ---------------------------------------------------------------------------
// One CTA per (tile, pair), kParFinalizeThreads threads.
constexpr int kParFinalizeThreads = 256;
__global__ void __launch_bounds__(kParFinalizeThreads) par_finalize_kernel(const __grid_constant__ ParParams p) {
  __shared__ ParTables tab;
  par_tables_to_smem(p.tab, tab);
  __shared__ float part[kParPartial];
  __shared__ float unit_re[kParFreq], unit_im[kParFreq], coh[kParFreq], wgt[kParFreq];
  __shared__ float theta[kParFreq], corr[kParPix];
  __shared__ float z_re[kParTH][kParWF], z_im[kParTH][kParWF];
  __shared__ float s_base, s_denom, s_conf, s_dx, s_dy, s_ramp;
  const int tile = blockIdx.x, pair = blockIdx.y, t = threadIdx.x;
  const float *src = p.partials + ((size_t)pair * kParTiles + tile) * p.n_stat_chunks * kParPartial;
  for (int r = t; r < kParPartial; r += blockDim.x) {
    float acc = 0.0f;
#pragma unroll 8
    for (int ch = 0; ch < p.n_stat_chunks; ++ch) acc += src[(size_t)ch * kParPartial + r];
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
  // PHAT correlation: irfft2(unit * coherence, s=(11,10)), separably: first
  // Z[y][kx] = sum_ky v e^{+i 2pi ky y / 11} ...
  if (t < kParTH * kParWF) {
    const int y = t / kParWF, kx = t % kParWF;
    float zr = 0.0f, zi = 0.0f;
#pragma unroll
    for (int ky = 0; ky < kParTH; ++ky) {
      const int my = (ky * y) % kParTH, f = ky * kParWF + kx;
      const float vr = unit_re[f] * coh[f], vi = unit_im[f] * coh[f];
      zr += vr * tab.ch[my] - vi * tab.shh[my];
      zi += vr * tab.shh[my] + vi * tab.ch[my];
    }
    z_re[y][kx] = zr;
    z_im[y][kx] = zi;
  }
  __syncthreads();
  // ... then the c2r rows over kx (imaginary parts of kx = 0 and 5 dropped)
  if (t < kParPix) {
    const int y = t / kParTW, x = t % kParTW;
    float acc = z_re[y][0] + ((x & 1) ? -z_re[y][kParWF - 1] : z_re[y][kParWF - 1]);
#pragma unroll
    for (int kx = 1; kx < kParWF - 1; ++kx) {
      const int mx = (kx * x) % kParTW;
      acc += 2.0f * (z_re[y][kx] * tab.cw[mx] - z_im[y][kx] * tab.sw[mx]);
    }
    corr[t] = acc * (1.0f / (float)(kParTH * kParTW));
  }
  __syncthreads();
  if (t < 32) {
    // first index of the maximum: each lane scans i = t, t + 32, ... in
    // order, then a shuffle tree keeps the larger value, the smaller index
    // on ties
    int best = t;
    float bv = corr[t];
    for (int i = t + 32; i < kParPix; i += 32)
      if (corr[i] > bv) {
        bv = corr[i];
        best = i;
      }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, best, o);
      if (ov > bv || (ov == bv && oi < best)) {
        bv = ov;
        best = oi;
      }
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
    if (t == 0) {
      s_dx = (float)(px >= (kParTW + 1) / 2 ? px - kParTW : px) + sub(xl, bv, xr);
      s_dy = (float)(py >= (kParTH + 1) / 2 ? py - kParTH : py) + sub(yu, bv, yd);
    }
  }
  __syncthreads();
  if (t < 32) {
    float acc = 0.0f;
    for (int f = t; f < kParFreq; f += 32) {
      const int ky = f / kParWF, kx = f % kParWF;
      const float ang = -(s_dy * tab.fy[ky] + s_dx * tab.fx[kx]);
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
    const float z = (s_conf - tab.thr[t]) / p.temperature;
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

// grid (tile, target, K chunk), 256 threads: the F images for the
// tensor-core prediction (spread over many SMs: building them is
// instruction-bound).
__global__ void __launch_bounds__(256) par_filter_kernel(const __grid_constant__ ParParams p) {
  __shared__ ParTables tab;
  __shared__ ParFilterSmem fs;
  par_tables_to_smem(p.tab, tab);
  par_build_filter(p, tab, blockIdx.x, blockIdx.y, blockIdx.z, blockIdx.z + 1, fs);
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

// Persistent tensor-core prediction.  Units (target, tile, chunk of 128
// channels) in that order; CTA c takes the contiguous range
// [c U / grid, (c + 1) U / grid), so F (per target and tile) changes at most
// a few times per CTA and stays resident in between.  Warp kParEpiWarps
// gathers the anchor tiles by TMA into two A buffers (one 64 x 10 x 11 box
// per anchor and channel half; slot order as par_box_y0 / par_box_x0) and
// issues the MMAs into two TMEM halves (lane 0); warps 0 .. 7 move D to the workspace (warp w:
// TMEM lanes 32 (w % 4) .., columns 64 (w / 4) ..).  Every wait is bounded;
// a failed wait stops the warp's loop and sets the device error.
__global__ void __launch_bounds__(kParPredThreads, 1)
    par_predict_mma_kernel(const __grid_constant__ CUtensorMap tm_act, const __grid_constant__ ParParams p) {
  extern __shared__ uint8_t par_smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(par_smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + ParMmaSmem::bars);
  uint64_t *a_full = bars, *b_full = bars + 2, *mma_done = bars + 3, *tmem_free = bars + 5;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + ParMmaSmem::tmem_slot);
  // set when one of this CTA's waits gives up, so the others stop too
  int *err = reinterpret_cast<int *>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nch = (p.C + 127) / 128;
  const int n_units = p.n_targets * kParTiles * nch;
  const int u0 = (int)((long long)blockIdx.x * n_units / gridDim.x);
  const int u1 = (int)((long long)(blockIdx.x + 1) * n_units / gridDim.x);
  const int n = u1 - u0;

  if (threadIdx.x == 0) {
    *err = 0;
    for (int i = 0; i < 2; ++i) {
      castdev::mbar_init(&a_full[i], 1);
      castdev::mbar_init(&mma_done[i], 1);
      castdev::mbar_init(&tmem_free[i], kParEpiWarps);
    }
    castdev::mbar_init(b_full, 1);
    castdev::fence_barrier_init();
  }
  if (warp == kParEpiWarps) {
    castdev::tmem_alloc(tmem_slot, 256);
    castdev::tmem_relinquish();
  }
  // K padding rows 110, 111, 222, 223 of both channel halves of both buffers
  // (the gather never writes them)
  for (int e = threadIdx.x; e < 2 * 2 * 4 * 8; e += blockDim.x) {
    const int buf = e / 64, h = (e / 32) % 2, r = (e / 8) % 4, c16 = e % 8;
    const int row = r < 2 ? kParPix + r : kParN + kParPix + (r - 2);
    *reinterpret_cast<uint4 *>(smem + ParMmaSmem::a + buf * 2 * kParAHalfBytes + h * kParAHalfBytes +
                               row * 128 + c16 * 16) = make_uint4(0u, 0u, 0u, 0u);
  }
  castdev::fence_proxy_async_smem();
  __syncthreads();
  castdev::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kParEpiWarps) {
    // ---- producer / MMA issuer ------------------------------------------
    const uint32_t sbase = castdev::smem_u32(smem);
    constexpr uint32_t idesc = castdev::make_idesc(1, 1, 1, 1, 0, 128, kParN);
    int g_issued[2] = {0, 0}, g_waited[2] = {0, 0};  // gathers per A buffer
    int f_loads = 0, f_waited = 0;
    // all of the issuer's work is lane 0's; the other lanes wait at the shuffles
    auto gather = [&](int k) {  // unit u0 + k into buffer k & 1: one box per anchor and channel half
      const int u = u0 + k, buf = k & 1;
      const int grp = u / nch, chunk = u % nch, tile = grp % kParTiles, tg = grp / kParTiles;
      const int pair = p.target_pair[tg], gy = tile / kParGW, gx = tile % kParGW;
      castdev::mbar_arrive_expect_tx(&a_full[buf], kParGatherBytes);
      for (int e = 0; e < 4; ++e) {
        const int h = e & 1, side = e >> 1;
        castdev::tma_load_4d(smem + ParMmaSmem::a + buf * 2 * kParAHalfBytes + h * kParAHalfBytes + side * kParN * 128,
                             &tm_act, &a_full[buf], chunk * 128 + h * 64, par_box_x0(gx), par_box_y0(gy),
                             side ? p.pair_right[pair] : p.pair_left[pair]);
      }
      ++g_issued[buf];
    };
    auto load_f = [&](int k) {
      const int grp = (u0 + k) / nch, tile = grp % kParTiles, tg = grp / kParTiles;
      castdev::mbar_arrive_expect_tx(b_full, kParFilterBytes);
      castdev::bulk_load(smem + ParMmaSmem::b, p.filters + ((size_t)tg * kParTiles + tile) * kParFilterBytes,
                         kParFilterBytes, b_full);
      ++f_loads;
    };
    bool ok = true;
    if (lane == 0 && n > 0) {
      castdev::tma_prefetch_desc(&tm_act);
      load_f(0);
      gather(0);
      if (n > 1) gather(1);
    }
    for (int k = 0; k < n && ok; ++k) {
      const int buf = k & 1;
      if (lane == 0) {
        if (k >= 1) {
          // unit k - 1's MMAs have completed: its A buffer takes unit k + 1,
          // and B may take a new F
          ok = castdev::mbar_wait(&mma_done[(k - 1) & 1], ((k - 1) >> 1) & 1, err);
          if (ok && k + 1 < n) gather(k + 1);
          if (ok && (u0 + k) / nch != (u0 + k - 1) / nch) load_f(k);
        }
        if (ok && f_waited < f_loads) {
          ok = castdev::mbar_wait(b_full, (f_loads - 1) & 1, err);
          f_waited = f_loads;
        }
        if (ok) {
          ok = castdev::mbar_wait(&a_full[buf], (k >> 1) & 1, err);
          ++g_waited[buf];
        }
        if (ok && k >= 2) ok = castdev::mbar_wait(&tmem_free[buf], ((k - 2) >> 1) & 1, err);
        if (ok) {
          castdev::tc_fence_after();
          const uint32_t a0 = sbase + ParMmaSmem::a + buf * 2 * kParAHalfBytes;
#pragma unroll 1
          for (int half = 0; half < 2; ++half) {  // F hi, then F lo
#pragma unroll
            for (int s = 0; s < kParK / 16; ++s) {
              const uint64_t ad = castdev::smem_desc_sw128(a0 + 2048 * s, kParAHalfBytes, 1024);
              const uint64_t bd = castdev::smem_desc_sw128(
                  sbase + ParMmaSmem::b + half * kParFHalfBytes + (s >> 2) * kParFChunkBytes + (s & 3) * 32,
                  16, 1024);
              castdev::mma_f16_ss(tmem + buf * kParN, ad, bd, idesc, (half | s) != 0);
            }
          }
          castdev::tc_commit(&mma_done[buf]);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    // nothing the TMA unit writes may be in flight when the block exits
    if (lane == 0) {
      for (int b2 = 0; b2 < 2; ++b2)
        if (g_issued[b2] > g_waited[b2]) castdev::mbar_wait_drain(&a_full[b2], (g_issued[b2] - 1) & 1, err);
      if (f_loads > f_waited) castdev::mbar_wait_drain(b_full, (f_loads - 1) & 1, err);
      if (n > 0) {  // the last MMAs have completed before TMEM is released
        castdev::mbar_wait_drain(&mma_done[(n - 1) & 1], ((n - 1) >> 1) & 1, err);
        if (n > 1) castdev::mbar_wait_drain(&mma_done[(n - 2) & 1], ((n - 2) >> 1) & 1, err);
      }
    }
    __syncwarp();
  } else {
    // ---- epilogue: D -> predicted tiles (fp32, workspace) -----------------
    const int q = warp & 3, colh = warp >> 2;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    for (int k = 0; k < n; ++k) {
      const int buf = k & 1, u = u0 + k;
      const int grp = u / nch, chunk = u % nch, tile = grp % kParTiles, tg = grp / kParTiles;
      int okw = 1;
      if (lane == 0) okw = castdev::mbar_wait(&mma_done[buf], (k >> 1) & 1, err);
      if (!__shfl_sync(0xffffffffu, okw, 0)) break;
      castdev::tc_fence_after();
      uint32_t v0[32], v1[32];
      const uint32_t col = tmem + lane_off + buf * kParN + 64 * colh;
      castdev::tmem_ld32(col, v0);
      if (colh == 0) castdev::tmem_ld32(col + 32, v1);
      else castdev::tmem_ld16(col + 32, *reinterpret_cast<uint32_t(*)[16]>(v1));
      castdev::tmem_wait_ld();
      castdev::tc_fence_before();
      __syncwarp();
      if (lane == 0) castdev::mbar_arrive(&tmem_free[buf]);
      const int c = chunk * 128 + q * 32 + lane;
      if (c < p.C) {
        float *dst = p.pred + (((size_t)tg * kParTiles + tile) * kParPix + 64 * colh) * p.C + c;
        const int n_cols = colh == 0 ? 64 : kParPix - 64;
#pragma unroll
        for (int j = 0; j < 32; ++j) dst[(size_t)j * p.C] = __uint_as_float(v0[j]);
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (32 + j < n_cols) dst[(size_t)(32 + j) * p.C] = __uint_as_float(v1[j]);
      }
    }
  }
  __syncthreads();
  if (warp == kParEpiWarps) {
    castdev::tc_fence_after();
    castdev::tmem_dealloc(tmem, 256);
  }
}

// ---------------------------------------------------------------------------
// Tensor-core statistics.  The windowed rfft2 of a tile is a fixed linear map
// of its 110 pixels, X[f] = sum_q win[q] x[q] e^{-i w_f . q}.  The input is
// real, so along kx = 0 and kx = 5 the bins of ky and 11 - ky are complex
// conjugates and bins (0, 0), (0, 5) are real: 110 independent real values.
// With the channels as M each anchor's independent spectrum is one GEMM,
// S[128 ch x 112] = A[128 ch x 112 px] Dft, the Dft columns (bf16 hi + lo)
//   2b, 2b+1  re, im of complex bin b: b < 44 -> (ky = b % 11, kx = 1 + b / 11),
//             44 <= b < 54 -> (ky = 1 + (b - 44) % 5, kx = b < 49 ? 0 : 5)
//   108, 109  bins (0, 0) and (0, 5) (real)
//   110, 111  zero.
// The per-bin products R conj(L), |R conj(L)| and their channel sums are the
// epilogue; the mirrored bins take the conjugate of their partner's sums.
constexpr int kParDftChunkBytes = kParN * 128;             // one 64-slot K chunk: 14336
constexpr int kParDftHalfBytes = 2 * kParDftChunkBytes;    // hi or lo: 28672
constexpr int kParDftBytes = 2 * kParDftHalfBytes;         // 57344
constexpr int kParCplx = 54;                               // independent complex bins
constexpr int kParStatVals = 3 * 48 + 24;                  // per-warp sums staged per item
constexpr int kParStatEpiWarps = 16;                       // 4 per TMEM lane quarter
constexpr int kParStatThreads = (kParStatEpiWarps + 1) * 32;  // + the TMA / MMA warp
constexpr int kParClasses = 9;

// Statistics: two A buffers, the class's Dft image, per-warp sums, then
// a_full[2], mma_done[2], tmem_free[2], b_full and the TMEM slot.
struct ParStatSmem {
  static constexpr int a = 0;
  static constexpr int b = 4 * kParAHalfBytes;
  static constexpr int wsum = b + kParDftBytes;             // [4 lane quarters][kParStatVals]
  static constexpr int bars = wsum + 4 * kParStatVals * 4;
  static constexpr int tmem_slot = bars + 7 * 8;
  static constexpr int total = tmem_slot + 8;
  static constexpr int alloc = total + 1024;
};
static_assert(ParStatSmem::alloc <= 227 * 1024, "statistics shared memory");
static_assert(ParStatSmem::bars % 8 == 0, "barrier alignment");

// (ky, kx) of independent complex bin b (layout above).
__device__ __forceinline__ void par_cplx_bin(int b, int &ky, int &kx) {
  if (b < 44) {
    ky = b % kParTH;
    kx = 1 + b / kParTH;
  } else {
    ky = 1 + (b - 44) % 5;
    kx = b < 49 ? 0 : kParWF - 1;
  }
}

// One halving step of a warp reduce-scatter: lanes with bit OFF set keep the
// upper half of v[0..N), the others the lower half, each adding its
// partner's copy of the kept half.
template <int N, int OFF>
__device__ __forceinline__ void par_rs_step(float *v, int lane) {
  constexpr int H = N / 2;
  const bool up = (lane & OFF) != 0;
#pragma unroll
  for (int i = 0; i < H; ++i) {
    const float send = up ? v[i] : v[H + i];
    const float keep = up ? v[H + i] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, OFF);
  }
}

// Warp sums of v[0..24): base = 12 [L&16] + 6 [L&8] + 3 [L&4]; stored by
// lanes with L & 3 == 0.
__device__ __forceinline__ void par_warp_sum24(float (&v)[24], int lane, float *out) {
  par_rs_step<24, 16>(v, lane);
  par_rs_step<12, 8>(v, lane);
  par_rs_step<6, 4>(v, lane);
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    v[i] += __shfl_xor_sync(0xffffffffu, v[i], 2);
    v[i] += __shfl_xor_sync(0xffffffffu, v[i], 1);
  }
  const int base = ((lane & 16) ? 12 : 0) + ((lane & 8) ? 6 : 0) + ((lane & 4) ? 3 : 0);
  if ((lane & 3) == 0) {
#pragma unroll
    for (int i = 0; i < 3; ++i) out[base + i] = v[i];
  }
}

// The class images depend only on the window and the tile geometry: the host
// builds them once per device into this array (or, inside a stream capture
// before that, as part of the captured work).
__device__ __align__(1024) uint8_t g_par_dft[kParClasses * kParDftBytes];

// grid (7, tile class), 256 threads, one thread per (column n, 8
// consecutive box slots): the class's Dft image, element (slot, n) = sum
// over the tile pixels (i, j) in that slot of win[i][j] e^{-i 2 pi (ky i / 11
// + kx j / 10)} (re or im by the column layout above), bf16 hi + lo, K-major
// with the 128-byte swizzle, hi at 0 and lo at kParDftHalfBytes.
__global__ void __launch_bounds__(256) par_dft_kernel(const __grid_constant__ ParParams p) {
  __shared__ uint32_t slotw[kParPix];
  __shared__ float ey_re[kParTH][kParTH], ey_im[kParTH][kParTH], ex_re[kParWF][kParTW], ex_im[kParWF][kParTW];
  __shared__ float win[kParPix];
  const int cls = blockIdx.y, t = threadIdx.x;
  const int t0 = par_class_tile(cls, 0);
  if (t < kParPix) {
    slotw[t] = par_slot_word(t0 / kParGW, t0 % kParGW, t);
    win[t] = p.tab.win[t];
  }
  if (t < kParTH * kParTH) {  // e^{-2 pi i ky i / 11}
    const int m = ((t / kParTH) * (t % kParTH)) % kParTH;
    double sv, cv;
    sincospi(2.0 * m / kParTH, &sv, &cv);
    ey_re[t / kParTH][t % kParTH] = (float)cv;
    ey_im[t / kParTH][t % kParTH] = (float)-sv;
  } else if (t < kParTH * kParTH + kParWF * kParTW) {  // e^{-2 pi i kx j / 10}
    const int e2 = t - kParTH * kParTH, m = ((e2 / kParTW) * (e2 % kParTW)) % kParTW;
    double sv, cv;
    sincospi(2.0 * m / kParTW, &sv, &cv);
    ex_re[e2 / kParTW][e2 % kParTW] = (float)cv;
    ex_im[e2 / kParTW][e2 % kParTW] = (float)-sv;
  }
  __syncthreads();
  const int e = blockIdx.x * blockDim.x + t;
  if (e >= kParN * (kParN / 8)) return;
  const int nn = e % kParN, g = e / kParN;  // a warp takes consecutive columns of one slot group
  int ky = 0, kx = 0;
  if (nn < 2 * kParCplx) par_cplx_bin(nn >> 1, ky, kx);
  else kx = nn == 2 * kParCplx ? 0 : kParWF - 1;
  const bool im = nn < 2 * kParCplx && (nn & 1);
  uint32_t hi[4], lo[4];
#pragma unroll
  for (int j = 0; j < 8; j += 2) {
    float v[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int slot = g * 8 + j + u;
      float val = 0.0f;
      if (nn < 2 * kParCplx + 2 && slot < kParPix) {
        const uint32_t sw = slotw[slot];
        const int rows = (sw >> 16) & 3, cols = (sw >> 20) & 3;
#pragma unroll
        for (int a = 0; a < 2; ++a)
#pragma unroll
          for (int b = 0; b < 2; ++b)
            if (a < rows && b < cols) {
              const int i = (sw >> (4 * a)) & 15, jj = (sw >> (8 + 4 * b)) & 15;
              // e^{-i(alpha + beta)}: re = cos(alpha + beta), im = -sin(alpha + beta)
              const float yr = ey_re[ky][i], yi = ey_im[ky][i], xr = ex_re[kx][jj], xi = ex_im[kx][jj];
              const float pr = yr * xr - yi * xi, pim = yr * xi + yi * xr;
              val += win[i * kParTW + jj] * (im ? pim : pr);
            }
      }
      v[u] = val;
    }
    const __nv_bfloat162 h2 = __floats2bfloat162_rn(v[0], v[1]);
    const float2 hf = __bfloat1622float2(h2);
    const __nv_bfloat162 l2 = __floats2bfloat162_rn(v[0] - hf.x, v[1] - hf.y);
    hi[j / 2] = *reinterpret_cast<const uint32_t *>(&h2);
    lo[j / 2] = *reinterpret_cast<const uint32_t *>(&l2);
  }
  const int kc = g / 8, grp = g % 8;
  uint8_t *img = p.dft + (size_t)cls * kParDftBytes;
  const int off = kc * kParDftChunkBytes + nn * 128 + ((grp ^ (nn & 7)) * 16);
  *reinterpret_cast<uint4 *>(img + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
  *reinterpret_cast<uint4 *>(img + kParDftHalfBytes + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
}

// Persistent statistics.  CTAs are assigned to tile classes
// (p.stat_cta_start); a class's CTAs take its items (tile of the class, pair,
// chunk of 128 channels) round-robin.  Each CTA loads its class's Dft image
// (par_dft_kernel) with one bulk copy.  Warp kParStatEpiWarps gathers the
// anchor tiles by TMA (one box per anchor and channel half) into two A
// buffers and issues the MMAs into two TMEM halves; warps 0 .. 15 form the
// per-bin products and channel sums (warp w: TMEM lanes 32 (w % 4) ..,
// column group w / 4, in 24-value butterflies (register budget: 17 warps);
// then the four lane quarters in order) and write the partials of each
// item's chunk.
__global__ void __launch_bounds__(kParStatThreads, 1)
    par_stats_mma_kernel(const __grid_constant__ CUtensorMap tm_act, const __grid_constant__ ParParams p) {
  extern __shared__ uint8_t par_smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(par_smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + ParStatSmem::bars);
  uint64_t *a_full = bars, *mma_done = bars + 2, *tmem_free = bars + 4, *b_full = bars + 6;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + ParStatSmem::tmem_slot);
  float *wsum = reinterpret_cast<float *>(smem + ParStatSmem::wsum);
  // set when one of this CTA's waits gives up, so the others stop too
  int *err = reinterpret_cast<int *>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nch = p.n_stat_chunks;

  // this CTA's class and its share of the class's items
  int cls = 0;
  while (cls + 1 < kParClasses && p.stat_cta_start[cls + 1] <= (int)blockIdx.x) ++cls;
  const int g_cls = p.stat_cta_start[cls + 1] - p.stat_cta_start[cls];
  const int first = blockIdx.x - p.stat_cta_start[cls];
  const int per_tile = p.n_pairs * nch;
  const int n_cls = par_class_tiles(cls) * per_tile;
  const int n = first < n_cls ? (n_cls - first + g_cls - 1) / g_cls : 0;
  auto item = [&](int k, int &tile, int &pair, int &chunk) {
    const int li = first + k * g_cls;
    tile = par_class_tile(cls, li / per_tile);
    pair = (li % per_tile) / nch;
    chunk = li % nch;
  };

  if (threadIdx.x == 0) {
    *err = 0;
    for (int i = 0; i < 2; ++i) {
      castdev::mbar_init(&a_full[i], 1);
      castdev::mbar_init(&mma_done[i], 1);
      castdev::mbar_init(&tmem_free[i], 1);
    }
    castdev::mbar_init(b_full, 1);
    castdev::fence_barrier_init();
  }
  if (warp == kParStatEpiWarps) {
    castdev::tmem_alloc(tmem_slot, 512);
    castdev::tmem_relinquish();
  }
  // K padding rows 110, 111, 222, 223 of both buffers (the gather never writes them)
  for (int e = threadIdx.x; e < 2 * 2 * 4 * 8; e += blockDim.x) {
    const int buf = e / 64, h = (e / 32) % 2, r = (e / 8) % 4, c16 = e % 8;
    const int row = r < 2 ? kParPix + r : kParN + kParPix + (r - 2);
    *reinterpret_cast<uint4 *>(smem + ParStatSmem::a + buf * 2 * kParAHalfBytes + h * kParAHalfBytes + row * 128 +
                               c16 * 16) = make_uint4(0u, 0u, 0u, 0u);
  }
  castdev::fence_proxy_async_smem();
  __syncthreads();
  castdev::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kParStatEpiWarps) {
    // ---- TMA / MMA issuer (lane 0) ------------------------------------------
    const uint32_t sbase = castdev::smem_u32(smem);
    constexpr uint32_t idesc = castdev::make_idesc(1, 1, 1, 1, 0, 128, kParN);
    int g_issued[2] = {0, 0}, g_waited[2] = {0, 0};
    auto gather = [&](int k) {
      int tile, pair, chunk;
      item(k, tile, pair, chunk);
      const int buf = k & 1, gy = tile / kParGW, gx = tile % kParGW;
      castdev::mbar_arrive_expect_tx(&a_full[buf], kParGatherBytes);
      for (int e = 0; e < 4; ++e) {
        const int h = e & 1, side = e >> 1;
        castdev::tma_load_4d(smem + ParStatSmem::a + buf * 2 * kParAHalfBytes + h * kParAHalfBytes + side * kParN * 128,
                             &tm_act, &a_full[buf], chunk * 128 + h * 64, par_box_x0(gx), par_box_y0(gy),
                             side ? p.pair_right[pair] : p.pair_left[pair]);
      }
      ++g_issued[buf];
    };
    bool ok = true;
    bool b_loaded = false;
    if (lane == 0 && n > 0) {
      castdev::tma_prefetch_desc(&tm_act);
      castdev::mbar_arrive_expect_tx(b_full, kParDftBytes);
      castdev::bulk_load(smem + ParStatSmem::b, p.dft + (size_t)cls * kParDftBytes, kParDftBytes, b_full);
      b_loaded = true;
      gather(0);
      if (n > 1) gather(1);
      ok = castdev::mbar_wait(b_full, 0, err);
      if (ok) b_loaded = false;
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    for (int k = 0; k < n && ok; ++k) {
      const int buf = k & 1;
      if (lane == 0) {
        if (k >= 1) {
          // unit k - 1's MMAs have completed: its A buffer takes item k + 1
          ok = castdev::mbar_wait(&mma_done[(k - 1) & 1], ((k - 1) >> 1) & 1, err);
          if (ok && k + 1 < n) gather(k + 1);
        }
        if (ok) {
          ok = castdev::mbar_wait(&a_full[buf], (k >> 1) & 1, err);
          ++g_waited[buf];
        }
        if (ok && k >= 2) ok = castdev::mbar_wait(&tmem_free[buf], ((k - 2) >> 1) & 1, err);
        if (ok) {
          castdev::tc_fence_after();
          const uint32_t a0 = sbase + ParStatSmem::a + buf * 2 * kParAHalfBytes;
#pragma unroll 1
          for (int side = 0; side < 2; ++side) {  // left anchor -> columns 0.., right -> 112..
#pragma unroll 1
            for (int half = 0; half < 2; ++half) {  // Dft hi, then Dft lo
#pragma unroll
              for (int s = 0; s < kParN / 16; ++s) {
                const uint64_t ad =
                    castdev::smem_desc_sw128(a0 + 2048 * (side * (kParN / 16) + s), kParAHalfBytes, 1024);
                const uint64_t bd = castdev::smem_desc_sw128(
                    sbase + ParStatSmem::b + half * kParDftHalfBytes + (s >> 2) * kParDftChunkBytes + (s & 3) * 32,
                    16, 1024);
                castdev::mma_f16_ss(tmem + buf * 2 * kParN + side * kParN, ad, bd, idesc, (half | s) != 0);
              }
            }
          }
          castdev::tc_commit(&mma_done[buf]);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    if (lane == 0) {  // nothing the TMA unit or the tensor core writes may be in flight at exit
      if (b_loaded) castdev::mbar_wait_drain(b_full, 0, err);
      for (int b2 = 0; b2 < 2; ++b2)
        if (g_issued[b2] > g_waited[b2]) castdev::mbar_wait_drain(&a_full[b2], (g_issued[b2] - 1) & 1, err);
      if (n > 0) castdev::mbar_wait_drain(&mma_done[(n - 1) & 1], ((n - 1) >> 1) & 1, err);
      if (n > 1) castdev::mbar_wait_drain(&mma_done[(n - 2) & 1], ((n - 2) >> 1) & 1, err);
    }
    __syncwarp();
  } else {
    // ---- epilogue warps (named barrier 1 over kParStatEpiWarps warps) ---------
    const int et = threadIdx.x;  // 0 .. kParStatEpiWarps * 32 - 1
    constexpr uint32_t kEpi = kParStatEpiWarps * 32;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    float *wout = wsum + (warp & 3) * kParStatVals;
    for (int k = 0; k < n; ++k) {
      const int buf = k & 1;
      int okw = 1;
      if (lane == 0) okw = castdev::mbar_wait(&mma_done[buf], (k >> 1) & 1, err);
      const bool done = __shfl_sync(0xffffffffu, okw, 0) != 0;
      castdev::tc_fence_after();
      const uint32_t tl = tmem + lane_off + buf * 2 * kParN;
      const int grp = warp >> 2;
      if (grp < 3) {  // complex bins 16 grp .. 16 grp + 15, 8 per butterfly
#pragma unroll 1
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t l[16], r[16];
          if (done) {
            castdev::tmem_ld16(tl + 32 * grp + 16 * hh, l);
            castdev::tmem_ld16(tl + kParN + 32 * grp + 16 * hh, r);
            castdev::tmem_wait_ld();
          }
          float v[24];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float lr = __uint_as_float(l[2 * j]), li = __uint_as_float(l[2 * j + 1]);
            const float rr = __uint_as_float(r[2 * j]), ri = __uint_as_float(r[2 * j + 1]);
            const float cre = rr * lr + ri * li, cim = ri * lr - rr * li;
            v[3 * j] = cre;
            v[3 * j + 1] = cim;
            v[3 * j + 2] = sqrtf(cre * cre + cim * cim);
          }
          par_warp_sum24(v, lane, wout + 48 * grp + 24 * hh);
        }
      } else {  // complex bins 48..53, then the real bins (0, 0) and (0, 5)
        uint32_t l[16], r[16];
        if (done) {
          castdev::tmem_ld16(tl + 96, l);
          castdev::tmem_ld16(tl + kParN + 96, r);
          castdev::tmem_wait_ld();
        }
        float v[24];
#pragma unroll
        for (int j = 0; j < 6; ++j) {
          const float lr = __uint_as_float(l[2 * j]), li = __uint_as_float(l[2 * j + 1]);
          const float rr = __uint_as_float(r[2 * j]), ri = __uint_as_float(r[2 * j + 1]);
          const float cre = rr * lr + ri * li, cim = ri * lr - rr * li;
          v[3 * j] = cre;
          v[3 * j + 1] = cim;
          v[3 * j + 2] = sqrtf(cre * cre + cim * cim);
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const float cre = __uint_as_float(r[12 + j]) * __uint_as_float(l[12 + j]);
          v[18 + 2 * j] = cre;
          v[19 + 2 * j] = sqrtf(cre * cre);
        }
        v[22] = v[23] = 0.0f;
        par_warp_sum24(v, lane, wout + 144);
      }
      castdev::tc_fence_before();
      castdev::named_bar_sync(1, kEpi);  // TMEM half read, per-quarter sums staged
      if (et == 0) castdev::mbar_arrive(&tmem_free[buf]);
      if (done) {
        int tile, pair, chunk;
        item(k, tile, pair, chunk);
        float *dst = p.partials + (((size_t)pair * kParTiles + tile) * nch + chunk) * kParPartial;
        for (int r = et; r < kParPartial; r += kEpi) {
          const int qn = r / kParFreq, f = r % kParFreq, ky = f / kParWF, kx = f % kParWF;
          int vi = -1;
          float sign = 1.0f;
          if (kx >= 1 && kx <= 4) {
            const int b = (kx - 1) * kParTH + ky;
            vi = b < 48 ? 48 * (b / 16) + 3 * (b % 16) + qn : 144 + 3 * (b - 48) + qn;
          } else if (ky == 0) {
            vi = qn == 1 ? -1 : 144 + 18 + (kx ? 2 : 0) + (qn ? 1 : 0);
          } else {
            const int kk = ky <= 5 ? ky : kParTH - ky;
            if (ky > 5 && qn == 1) sign = -1.0f;
            const int b = 44 + (kx ? 5 : 0) + kk - 1;
            vi = b < 48 ? 48 * (b / 16) + 3 * (b % 16) + qn : 144 + 3 * (b - 48) + qn;
          }
          float acc = 0.0f;
          if (vi >= 0) {
#pragma unroll
            for (int w = 0; w < 4; ++w) acc += wsum[w * kParStatVals + vi];
          }
          dst[r] = sign * acc;
        }
      }
      castdev::named_bar_sync(1, kEpi);  // sums read before the next item's staging
    }
  }
  __syncthreads();
  if (warp == kParStatEpiWarps) {
    castdev::tc_fence_after();
    castdev::tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// grid (HW, n_targets); each thread handles 4 channels.
// The routing transport's mean affinities (stats tail): each used pair's
// mean over its 18 x 66 affinities, and the mean over the targets of their
// pair's affinities, summed in double in a fixed order by one CTA.
__device__ void par_mean_affinity(const ParParams &p) {
  __shared__ double red[256 / 32];
  __shared__ double pair_sum[kParMaxPairs];
  constexpr int per = kParTiles * (2 * kParFreq + 5), g0 = kParTiles * (kParFreq + 1);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int pr = 0; pr < p.n_pairs; ++pr) {
    const float *g = p.stats + (size_t)pr * per + g0;
    double s = 0.0;
    for (int i = threadIdx.x; i < kParTiles * kParFreq; i += blockDim.x) s += (double)g[i];
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
      double t = 0.0;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
      pair_sum[pr] = t;
      p.stats[(size_t)kParMaxPairs * per + pr] = (float)(t / (kParTiles * kParFreq));
    }
    __syncthreads();
  }
  if (threadIdx.x == 0 && p.n_targets > 0) {
    double t = 0.0;
    for (int tg = 0; tg < p.n_targets; ++tg) t += pair_sum[p.target_pair[tg]];
    p.stats[(size_t)kParMaxPairs * per + kParMaxPairs] =
        (float)(t / ((double)p.n_targets * kParTiles * kParFreq));
  }
}

__global__ void __launch_bounds__(256) par_ola_kernel(const ParParams p) {
  if (p.stats && blockIdx.x == 0 && blockIdx.y == 0) par_mean_affinity(p);
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
