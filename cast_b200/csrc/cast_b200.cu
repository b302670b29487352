// Single translation unit of libcast_b200.so: the extern "C" entry points
// declared in include/cast_b200.h and the host-side launch logic.
#include <algorithm>
#include <cstdarg>
#include <cstdlib>
#include <cmath>
#include <functional>
#include <map>
#include <mutex>
#include <queue>
#include <vector>

#include "common.cuh"
#include "select_quant.cuh"
#include "attention.cuh"
#include "par.cuh"
#include "compact.cuh"
#include "barycentric.cuh"
#include "swap_router.cuh"

namespace cast {

static thread_local std::string g_last_error;

void set_error(const std::string &msg) { g_last_error = msg; }

int fail(int status, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

int current_device_sm100(int *num_sms) {
  int dev = 0;
  CAST_CUDA_TRY(cudaGetDevice(&dev));
  int major = 0, minor = 0;
  CAST_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
  CAST_CUDA_TRY(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev));
  if (major != 10 || minor != 0)
    return fail(CAST_ERR_NO_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a", dev,
                major, minor);
  if (num_sms) CAST_CUDA_TRY(cudaDeviceGetAttribute(num_sms, cudaDevAttrMultiProcessorCount, dev));
  return CAST_OK;
}

int get_encode_tiled(EncodeTiledFn *fn) {
  static EncodeTiledFn cached = nullptr;
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    if (err == cudaSuccess && q == cudaDriverEntryPointSuccess)
      cached = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  if (!cached)
    return fail(CAST_ERR_CUDA, "cuTensorMapEncodeTiled unavailable: %s", cudaGetErrorString(err));
  *fn = cached;
  return CAST_OK;
}

int make_map_3d(CUtensorMap *map, const void *base, CUtensorMapDataType dtype, int elem_bytes,
                uint64_t d0, uint64_t d1, uint64_t d2, uint32_t box0, uint32_t box1,
                CUtensorMapSwizzle swizzle) {
  EncodeTiledFn enc;
  int st = get_encode_tiled(&enc);
  if (st) return st;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {d0 * elem_bytes, d0 * d1 * elem_bytes};
  cuuint32_t box[3] = {box0, box1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, dtype, 3, const_cast<void *>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(CAST_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return CAST_OK;
}

// 4-D tiled map over a dense [d3][d2][d1][d0] tensor, box (box0, box1, box2, 1).
// A 4-D map with explicit byte strides of dims 1..3 (multiples of 16).
int make_map_4d_strided(CUtensorMap *map, const void *base, CUtensorMapDataType dtype,
                        const uint64_t (&dims)[4], const uint64_t (&strides)[3], uint32_t box0,
                        uint32_t box1, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn enc;
  int st = get_encode_tiled(&enc);
  if (st) return st;
  cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
  cuuint64_t str[3] = {strides[0], strides[1], strides[2]};
  cuuint32_t box[4] = {box0, box1, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, dtype, 4, const_cast<void *>(base), d, str, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(CAST_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return CAST_OK;
}

int make_map_4d(CUtensorMap *map, const void *base, CUtensorMapDataType dtype, int elem_bytes,
                uint64_t d0, uint64_t d1, uint64_t d2, uint64_t d3, uint32_t box0, uint32_t box1,
                uint32_t box2, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn enc;
  int st = get_encode_tiled(&enc);
  if (st) return st;
  cuuint64_t dims[4] = {d0, d1, d2, d3};
  cuuint64_t strides[3] = {d0 * elem_bytes, d0 * d1 * elem_bytes, d0 * d1 * d2 * elem_bytes};
  cuuint32_t box[4] = {box0, box1, box2, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, dtype, 4, const_cast<void *>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(CAST_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return CAST_OK;
}

}  // namespace cast

using namespace cast;

// ===========================================================================
// status / version
// ===========================================================================
extern "C" const char *cast_status_string(int status) {
  switch (status) {
    case CAST_OK: return "CAST_OK";
    case CAST_ERR_INVALID_ARGUMENT: return "CAST_ERR_INVALID_ARGUMENT";
    case CAST_ERR_UNSUPPORTED: return "CAST_ERR_UNSUPPORTED";
    case CAST_ERR_ALIGNMENT: return "CAST_ERR_ALIGNMENT";
    case CAST_ERR_WORKSPACE: return "CAST_ERR_WORKSPACE";
    case CAST_ERR_CUDA: return "CAST_ERR_CUDA";
    case CAST_ERR_DEVICE_TIMEOUT: return "CAST_ERR_DEVICE_TIMEOUT";
    case CAST_ERR_NO_DEVICE: return "CAST_ERR_NO_DEVICE";
    default: return "CAST_ERR_UNKNOWN";
  }
}

extern "C" const char *cast_last_error_message(void) { return g_last_error.c_str(); }

extern "C" int cast_version(void) { return 100; }

extern "C" int cast_device_error(cast_stream_t stream) {
  CAST_CUDA_TRY(cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream)));
  int v = 0, zero = 0;
  CAST_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_cast_device_error, sizeof(int)));
  CAST_CUDA_TRY(cudaMemcpyToSymbol(g_cast_device_error, &zero, sizeof(int)));
  if (v) return fail(v, "device-side error: %s (a bounded wait gave up, or an index was out of range)",
                    cast_status_string(v));
  return CAST_OK;
}

// One CTA: an mbarrier expecting one arrival, which thread 0 makes only when
// `arrive`; every thread then waits on it through the library's bounded wait
// with the given limit.  Without the arrival the wait gives up, sets the
// device error word and the kernel returns normally.
__global__ void selftest_bounded_wait_kernel(int arrive, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int cta_abort;
  if (threadIdx.x == 0) {
    cta_abort = 0;
    castdev::mbar_init(&bar, 1);
    castdev::fence_barrier_init();
  }
  __syncthreads();
  if (arrive && threadIdx.x == 0) castdev::mbar_arrive(&bar);
  castdev::mbar_wait(&bar, 0, &cta_abort, limit_ns);
}

extern "C" int cast_selftest_bounded_wait(int arrive, int limit_us, cast_stream_t stream) {
  if (limit_us <= 0 || limit_us > 1000000)
    return fail(CAST_ERR_INVALID_ARGUMENT, "limit_us %d (1..1000000)", limit_us);
  int st = current_device_sm100(nullptr);
  if (st) return st;
  selftest_bounded_wait_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      arrive, (unsigned long long)limit_us * 1000ull);
  CAST_CUDA_TRY(cudaGetLastError());
  return CAST_OK;
}

// ===========================================================================
// RCSA selection + quantisation
// ===========================================================================
static size_t sq_pooled_bytes(int B, int H, int nqb, int nkb, int D) {
  return align_up((size_t)B * H * (nqb + nkb) * D * sizeof(double), 256);
}
static size_t sq_rms_bytes(int B, int H, int nqb, int nkb) {
  return align_up((size_t)B * H * (nqb + nkb) * sizeof(float), 256);
}

extern "C" size_t cast_rcsa_select_quant_workspace_bytes(int B, int H, int Lq, int Lk, int D,
                                                         int block_size) {
  if (B <= 0 || H <= 0 || Lq <= 0 || Lk <= 0 || D <= 0 || block_size <= 0) return 0;
  const int nqb = ceil_div(Lq, block_size), nkb = ceil_div(Lk, block_size);
  // pooled vectors, block RMS, and the q/k scales when the caller passes none
  return sq_pooled_bytes(B, H, nqb, nkb, D) + sq_rms_bytes(B, H, nqb, nkb) +
         2 * align_up((size_t)B * H * (nqb + nkb) * sizeof(float), 256) +
         align_up((size_t)B * H * (nqb + nkb), 256);  // need flags of the auto policy's code pass
}

extern "C" int cast_rcsa_select_quant(const void *q, const void *k, const void *v,
                                      const uint8_t *q_valid, const uint8_t *k_valid, int B, int H,
                                      int Lq, int Lk, int D, int block_size, int budget, int rule,
                                      int32_t *sel_idx, int32_t *sel_cnt, int8_t *q_codes,
                                      float *q_scales, int8_t *k_codes, float *k_scales,
                                      int8_t *v_codes, float *v_scales, uint8_t *qk_mode,
                                      int policy, float int8_tolerance, double *pooled,
                                      void *workspace, size_t workspace_bytes,
                                      cast_stream_t stream) {
  if (!q || !k || !sel_idx || !sel_cnt)
    return fail(CAST_ERR_INVALID_ARGUMENT, "q, k, sel_idx and sel_cnt are required");
  if (B <= 0 || H <= 0 || Lq <= 0 || Lk <= 0 || block_size <= 0 || budget < 0)
    return fail(CAST_ERR_INVALID_ARGUMENT, "non-positive size (B=%d H=%d Lq=%d Lk=%d block=%d budget=%d)",
                B, H, Lq, Lk, block_size, budget);
  if (rule != CAST_RULE_BUDGET_CAUSAL) return fail(CAST_ERR_INVALID_ARGUMENT, "unknown rule %d", rule);
  if (policy < CAST_POLICY_BF16 || policy > CAST_POLICY_AUTO)
    return fail(CAST_ERR_INVALID_ARGUMENT, "unknown precision policy %d", policy);
  if (D != 64 && D != 128) return fail(CAST_ERR_UNSUPPORTED, "head_dim %d (supported: 64, 128)", D);
  const int nqb = ceil_div(Lq, block_size), nkb = ceil_div(Lk, block_size);
  if (nkb < nqb) return fail(CAST_ERR_INVALID_ARGUMENT, "fewer key blocks (%d) than query blocks (%d)", nkb, nqb);
  if (budget > 256) return fail(CAST_ERR_UNSUPPORTED, "budget %d > 256", budget);
  if (!aligned16(q) || !aligned16(k) || (v && !aligned16(v)))
    return fail(CAST_ERR_ALIGNMENT, "q/k/v must be 16-byte aligned");
  if ((q_codes && !aligned16(q_codes)) || (k_codes && !aligned16(k_codes)) ||
      (v_codes && !aligned16(v_codes)))
    return fail(CAST_ERR_ALIGNMENT, "code buffers must be 16-byte aligned");
  if (qk_mode && policy == CAST_POLICY_AUTO && (!q_codes || !k_codes))
    return fail(CAST_ERR_INVALID_ARGUMENT, "the auto policy needs q_codes and k_codes");
  const size_t need = cast_rcsa_select_quant_workspace_bytes(B, H, Lq, Lk, D, block_size);
  if (!workspace || workspace_bytes < need)
    return fail(CAST_ERR_WORKSPACE, "workspace %zu bytes < required %zu", workspace_bytes, need);
  int n_sms = 0;
  int st = current_device_sm100(&n_sms);
  if (st) return st;

  uint8_t *ws = static_cast<uint8_t *>(workspace);
  double *pooled_ws = reinterpret_cast<double *>(ws);
  ws += sq_pooled_bytes(B, H, nqb, nkb, D);
  float *rms = reinterpret_cast<float *>(ws);
  ws += sq_rms_bytes(B, H, nqb, nkb);
  float *qs = q_scales ? q_scales : reinterpret_cast<float *>(ws);
  ws += align_up((size_t)B * H * (nqb + nkb) * sizeof(float), 256);
  float *ks = k_scales ? k_scales : reinterpret_cast<float *>(ws);
  ws += align_up((size_t)B * H * (nqb + nkb) * sizeof(float), 256);
  uint8_t *need_flags = ws;
  double *pooled_out = pooled ? pooled : pooled_ws;

  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int nb_total = nqb + nkb + ((v && v_codes) ? nkb : 0);
  dim3 grid(nb_total, B * H);
  const __nv_bfloat16 *qb = static_cast<const __nv_bfloat16 *>(q);
  const __nv_bfloat16 *kb = static_cast<const __nv_bfloat16 *>(k);
  const __nv_bfloat16 *vb = static_cast<const __nv_bfloat16 *>(v);
  // the masked variant only when a validity mask is given
  const bool masked = q_valid || k_valid;
  // Few blocks (one CTA per SM covers them all: a head-sharded call on many
  // GPUs) that fit in shared memory (unmasked, codes wanted, no V codes):
  // kernel 1s stages each block and writes every block's codes from there,
  // one read of Q and K in all.  With more blocks than SMs its one CTA per
  // SM keeps too few reads in flight (config 2, 24 heads: 92 against 87 us
  // int8), so the two-pass kernel runs.  Otherwise, under the auto policy,
  // codes only for the blocks the int8 query blocks read, written after the
  // selection (kernel 3); V codes keep the fused pass.
  const size_t staged_bytes = castk::staged_block_bytes(block_size, D);
  const bool staged = staged_bytes > 0 && !masked && !v_codes && q_codes && k_codes &&
                      (long long)B * H * (nqb + nkb) <= n_sms;
  const bool lazy = !staged && policy == CAST_POLICY_AUTO && qk_mode && !v_codes;
  int8_t *qc1 = lazy ? nullptr : q_codes, *kc1 = lazy ? nullptr : k_codes;
  uint8_t *nf = lazy ? need_flags : nullptr;
  if (staged) {
    static std::once_flag staged_once;
    static cudaError_t staged_err = cudaSuccess;
    std::call_once(staged_once, [] {
      // the opt-in limit covers static and dynamic shared memory together
      constexpr int kDyn = 227 * 1024 - (int)castk::kStagedStaticBytes;
      staged_err = cudaFuncSetAttribute(castk::pool_quant_staged_kernel<128>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, kDyn);
      if (staged_err == cudaSuccess)
        staged_err = cudaFuncSetAttribute(castk::pool_quant_staged_kernel<64>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, kDyn);
    });
    CAST_CUDA_TRY(staged_err);
    dim3 gs(nqb + nkb, B * H);
    if (D == 128)
      castk::pool_quant_staged_kernel<128><<<gs, 256, staged_bytes, s>>>(qb, kb, Lq, Lk, block_size, nqb, nkb,
                                                                        q_codes, qs, k_codes, ks, pooled_out, rms);
    else
      castk::pool_quant_staged_kernel<64><<<gs, 128, staged_bytes, s>>>(qb, kb, Lq, Lk, block_size, nqb, nkb,
                                                                       q_codes, qs, k_codes, ks, pooled_out, rms);
  } else if (D == 128 && !masked)
    castk::pool_quant_kernel<128, false><<<grid, 256, 0, s>>>(qb, kb, vb, q_valid, k_valid, Lq, Lk, block_size,
                                                              nqb, nkb, qc1, qs, kc1, ks, v_codes,
                                                              v_scales, pooled_out, rms, nf);
  else if (D == 128)
    castk::pool_quant_kernel<128, true><<<grid, 256, 0, s>>>(qb, kb, vb, q_valid, k_valid, Lq, Lk, block_size,
                                                             nqb, nkb, qc1, qs, kc1, ks, v_codes,
                                                             v_scales, pooled_out, rms, nf);
  else if (!masked)
    castk::pool_quant_kernel<64, false><<<grid, 128, 0, s>>>(qb, kb, vb, q_valid, k_valid, Lq, Lk, block_size,
                                                             nqb, nkb, qc1, qs, kc1, ks, v_codes,
                                                             v_scales, pooled_out, rms, nf);
  else
    castk::pool_quant_kernel<64, true><<<grid, 128, 0, s>>>(qb, kb, vb, q_valid, k_valid, Lq, Lk, block_size,
                                                            nqb, nkb, qc1, qs, kc1, ks, v_codes,
                                                            v_scales, pooled_out, rms, nf);
  CAST_CUDA_TRY(cudaGetLastError());
  const int keep = std::min(budget, nkb - nqb);
  const int maxdeg = keep + nqb;
  // Selection kernel shared memory: sort keys over the next power of two of
  // the history blocks, key-block RMS and scales, and (when they fit in
  // 160 KB) the history's pooled vectors staged by asynchronous copies.
  const int nhist = nkb - nqb;
  int pw = 1;
  while (pw < nhist) pw <<= 1;
  const size_t dsm_base = (sizeof(double) + sizeof(int32_t)) * pw + 2 * sizeof(float) * nkb + 16;
  const size_t stage_bytes = (size_t)nhist * D * sizeof(double);
  const bool stage_k = stage_bytes <= 160 * 1024;
  const size_t dsm = dsm_base + (stage_k ? stage_bytes : 0);
  if (dsm > 200 * 1024) return fail(CAST_ERR_UNSUPPORTED, "too many key blocks (%d)", nkb);
  static std::once_flag bsel_once;
  static cudaError_t bsel_err = cudaSuccess;
  std::call_once(bsel_once, [] {
    bsel_err = cudaFuncSetAttribute(castk::budget_select_kernel<128>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (bsel_err == cudaSuccess)
      bsel_err = cudaFuncSetAttribute(castk::budget_select_kernel<64>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  });
  CAST_CUDA_TRY(bsel_err);
  dim3 g2(nqb, B * H);
  if (D == 128)
    castk::budget_select_kernel<128><<<g2, 256, dsm, s>>>(pooled_out, rms, qs, ks, nqb, nkb,
                                                          budget, maxdeg, sel_idx, sel_cnt,
                                                          qk_mode, policy, int8_tolerance, stage_k, nf);
  else
    castk::budget_select_kernel<64><<<g2, 256, dsm, s>>>(pooled_out, rms, qs, ks, nqb, nkb,
                                                         budget, maxdeg, sel_idx, sel_cnt, qk_mode,
                                                         policy, int8_tolerance, stage_k, nf);
  CAST_CUDA_TRY(cudaGetLastError());
  if (lazy) {
    const int g3 = B * H * (nqb + nkb);  // one CTA per block; unmarked ones exit at once
#define CAST_QUANT_NEEDED(DD, MM, TT)                                                                \
  castk::quant_needed_kernel<DD, MM><<<g3, TT, 0, s>>>(qb, kb, q_valid, k_valid, Lq, Lk, block_size, \
                                                       nqb, nkb, B * H, need_flags, q_codes, qs,     \
                                                       k_codes, ks)
    if (D == 128 && !masked)
      CAST_QUANT_NEEDED(128, false, 256);
    else if (D == 128)
      CAST_QUANT_NEEDED(128, true, 256);
    else if (!masked)
      CAST_QUANT_NEEDED(64, false, 128);
    else
      CAST_QUANT_NEEDED(64, true, 128);
#undef CAST_QUANT_NEEDED
    CAST_CUDA_TRY(cudaGetLastError());
  }
  return CAST_OK;
}

// ===========================================================================
// Compact-path selection
// ===========================================================================
extern "C" size_t cast_compact_select_workspace_bytes(int B, int H, int n_blocks, int block_size,
                                                      int D) {
  if (B <= 0 || H <= 0 || n_blocks <= 0 || block_size <= 0 || D <= 0) return 0;
  const int L = n_blocks * block_size;
  return cast_rcsa_select_quant_workspace_bytes(B, H, L, L, D, block_size);
}

extern "C" int cast_compact_select(const void *q, const void *k, const uint8_t *valid, int B, int H,
                                   int n_blocks, int block_size, int D, int nh, int nw,
                                   const int32_t *row_degrees, int max_degree, int32_t *sel_idx,
                                   int32_t *sel_cnt, int8_t *q_codes, float *q_scales,
                                   int8_t *k_codes, float *k_scales, uint8_t *qk_mode, int policy,
                                   float int8_tolerance, double *pooled, void *workspace,
                                   size_t workspace_bytes, cast_stream_t stream) {
  if (!q || !k || !valid || !row_degrees || !sel_idx || !sel_cnt)
    return fail(CAST_ERR_INVALID_ARGUMENT, "q, k, valid, row_degrees, sel_idx and sel_cnt are required");
  if (B <= 0 || H <= 0 || n_blocks <= 0 || block_size <= 0 || nh <= 0 || nw <= 0 ||
      max_degree <= 0 || max_degree > n_blocks || n_blocks % (nh * nw))
    return fail(CAST_ERR_INVALID_ARGUMENT,
                "bad sizes (B=%d H=%d blocks=%d block=%d grid %dx%d max_degree=%d)", B, H, n_blocks,
                block_size, nh, nw, max_degree);
  if (policy < CAST_POLICY_BF16 || policy > CAST_POLICY_AUTO)
    return fail(CAST_ERR_INVALID_ARGUMENT, "unknown precision policy %d", policy);
  if (D != 64 && D != 128) return fail(CAST_ERR_UNSUPPORTED, "head_dim %d (supported: 64, 128)", D);
  if (!aligned16(q) || !aligned16(k)) return fail(CAST_ERR_ALIGNMENT, "q/k must be 16-byte aligned");
  if ((q_codes && !aligned16(q_codes)) || (k_codes && !aligned16(k_codes)))
    return fail(CAST_ERR_ALIGNMENT, "code buffers must be 16-byte aligned");
  if (qk_mode && policy != CAST_POLICY_BF16 && (!q_codes || !k_codes || !q_scales || !k_scales))
    return fail(CAST_ERR_INVALID_ARGUMENT, "int8 policies need q/k codes and scales");
  const int nb = n_blocks, L = nb * block_size;
  const size_t need = cast_compact_select_workspace_bytes(B, H, nb, block_size, D);
  if (!workspace || workspace_bytes < need)
    return fail(CAST_ERR_WORKSPACE, "workspace %zu bytes < required %zu", workspace_bytes, need);
  int st = current_device_sm100(nullptr);
  if (st) return st;
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  double *pooled_ws = reinterpret_cast<double *>(ws);
  ws += sq_pooled_bytes(B, H, nb, nb, D);
  float *rms = reinterpret_cast<float *>(ws);
  ws += sq_rms_bytes(B, H, nb, nb);
  float *qs = q_scales ? q_scales : reinterpret_cast<float *>(ws);
  ws += align_up((size_t)B * H * 2 * nb * sizeof(float), 256);
  float *ks = k_scales ? k_scales : reinterpret_cast<float *>(ws);
  ws += align_up((size_t)B * H * 2 * nb * sizeof(float), 256);
  uint8_t *need_flags = ws;
  double *pooled_out = pooled ? pooled : pooled_ws;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const __nv_bfloat16 *qb = static_cast<const __nv_bfloat16 *>(q);
  const __nv_bfloat16 *kb = static_cast<const __nv_bfloat16 *>(k);
  // pooled (masked) means, block RMS and scales; codes in the same pass for
  // the int8 policy, after the selection for the auto policy
  const bool lazy = policy == CAST_POLICY_AUTO && qk_mode;
  const bool codes_now = policy == CAST_POLICY_INT8 && qk_mode;
  int8_t *qc1 = codes_now ? q_codes : nullptr, *kc1 = codes_now ? k_codes : nullptr;
  uint8_t *nf = lazy ? need_flags : nullptr;
  dim3 grid(2 * nb, B * H);
  if (D == 128)
    castk::pool_quant_kernel<128, true><<<grid, 256, 0, s>>>(qb, kb, nullptr, valid, valid, L, L, block_size,
                                                             nb, nb, qc1, qs, kc1, ks, nullptr, nullptr,
                                                             pooled_out, rms, nf);
  else
    castk::pool_quant_kernel<64, true><<<grid, 128, 0, s>>>(qb, kb, nullptr, valid, valid, L, L, block_size,
                                                            nb, nb, qc1, qs, kc1, ks, nullptr, nullptr,
                                                            pooled_out, rms, nf);
  CAST_CUDA_TRY(cudaGetLastError());
  int pw = 1;
  while (pw < nb) pw <<= 1;
  const size_t dsm_base = (sizeof(double) + sizeof(int32_t)) * pw + 2 * sizeof(float) * nb + 16;
  const size_t stage_bytes = (size_t)nb * D * sizeof(double);
  const bool stage_k = stage_bytes <= 160 * 1024;
  const size_t dsm = dsm_base + (stage_k ? stage_bytes : 0);
  if (dsm > 200 * 1024) return fail(CAST_ERR_UNSUPPORTED, "too many compact blocks (%d)", nb);
  static std::once_flag csel_once;
  static cudaError_t csel_err = cudaSuccess;
  std::call_once(csel_once, [] {
    csel_err = cudaFuncSetAttribute(castk::compact_select_kernel<128>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (csel_err == cudaSuccess)
      csel_err = cudaFuncSetAttribute(castk::compact_select_kernel<64>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  });
  CAST_CUDA_TRY(csel_err);
  dim3 g2(nb, B * H);
  if (D == 128)
    castk::compact_select_kernel<128><<<g2, 256, dsm, s>>>(pooled_out, rms, qs, ks, nb, nh, nw, row_degrees,
                                                           max_degree, sel_idx, sel_cnt, qk_mode, policy,
                                                           int8_tolerance, stage_k, nf);
  else
    castk::compact_select_kernel<64><<<g2, 256, dsm, s>>>(pooled_out, rms, qs, ks, nb, nh, nw, row_degrees,
                                                          max_degree, sel_idx, sel_cnt, qk_mode, policy,
                                                          int8_tolerance, stage_k, nf);
  CAST_CUDA_TRY(cudaGetLastError());
  if (lazy) {
    const int g3 = B * H * 2 * nb;
    if (D == 128)
      castk::quant_needed_kernel<128, true><<<g3, 256, 0, s>>>(qb, kb, valid, valid, L, L, block_size, nb,
                                                               nb, B * H, need_flags, q_codes, qs, k_codes, ks);
    else
      castk::quant_needed_kernel<64, true><<<g3, 128, 0, s>>>(qb, kb, valid, valid, L, L, block_size, nb,
                                                              nb, B * H, need_flags, q_codes, qs, k_codes, ks);
    CAST_CUDA_TRY(cudaGetLastError());
  }
  return CAST_OK;
}

// ===========================================================================
// TABA selection
// ===========================================================================
extern "C" size_t cast_taba_select_workspace_bytes(int B, int H, int T, int Hl, int Wl, int D,
                                                   int tt, int th, int tw) {
  if (B <= 0 || H <= 0 || T <= 0 || Hl <= 0 || Wl <= 0 || D <= 0 || tt <= 0 || th <= 0 || tw <= 0)
    return 0;
  const size_t nblocks = (size_t)ceil_div(T, tt) * ceil_div(Hl, th) * ceil_div(Wl, tw);
  return align_up((size_t)B * H * 2 * nblocks * D * sizeof(double), 256);
}

extern "C" int cast_taba_select(const void *q, const void *k, int B, int H, int T, int Hl, int Wl,
                                int D, int tt, int th, int tw, const int32_t *row_degrees,
                                int max_degree, int32_t *sel_idx, int32_t *sel_cnt,
                                double *scores, void *workspace, size_t workspace_bytes,
                                cast_stream_t stream) {
  if (!q || !k || !row_degrees || !sel_idx || !sel_cnt)
    return fail(CAST_ERR_INVALID_ARGUMENT, "q, k, row_degrees, sel_idx, sel_cnt are required");
  if (B <= 0 || H <= 0 || T <= 0 || Hl <= 0 || Wl <= 0 || tt <= 0 || th <= 0 || tw <= 0)
    return fail(CAST_ERR_INVALID_ARGUMENT, "non-positive size");
  if (D != 64 && D != 128) return fail(CAST_ERR_UNSUPPORTED, "head_dim %d (supported: 64, 128)", D);
  const int nh = ceil_div(Hl, th), nw = ceil_div(Wl, tw), nt = ceil_div(T, tt);
  const int nblocks = nt * nh * nw;
  if (max_degree <= 0 || max_degree > nblocks)
    return fail(CAST_ERR_INVALID_ARGUMENT, "max_degree %d outside [1, %d]", max_degree, nblocks);
  if (!aligned16(q) || !aligned16(k)) return fail(CAST_ERR_ALIGNMENT, "q/k must be 16-byte aligned");
  const size_t need = cast_taba_select_workspace_bytes(B, H, T, Hl, Wl, D, tt, th, tw);
  if (!workspace || workspace_bytes < need)
    return fail(CAST_ERR_WORKSPACE, "workspace %zu bytes < required %zu", workspace_bytes, need);
  const size_t dsm = 2 * sizeof(double) * nblocks + nblocks + 16;
  if (dsm > 48 * 1024) return fail(CAST_ERR_UNSUPPORTED, "too many blocks (%d)", nblocks);
  int st = current_device_sm100(nullptr);
  if (st) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  double *pooled = static_cast<double *>(workspace);
  dim3 grid(2 * nblocks, B * H);
  const __nv_bfloat16 *qb = static_cast<const __nv_bfloat16 *>(q);
  const __nv_bfloat16 *kb = static_cast<const __nv_bfloat16 *>(k);
  if (D == 128)
    castk::pool_grid_kernel<128><<<grid, 256, 0, s>>>(qb, kb, T, Hl, Wl, tt, th, tw, nh, nw, nblocks, pooled);
  else
    castk::pool_grid_kernel<64><<<grid, 128, 0, s>>>(qb, kb, T, Hl, Wl, tt, th, tw, nh, nw, nblocks, pooled);
  CAST_CUDA_TRY(cudaGetLastError());
  dim3 g2(nblocks, B * H);
  if (D == 128)
    castk::taba_select_kernel<128><<<g2, 128, dsm, s>>>(pooled, nblocks, nh, nw, row_degrees,
                                                        max_degree, sel_idx, sel_cnt, scores);
  else
    castk::taba_select_kernel<64><<<g2, 128, dsm, s>>>(pooled, nblocks, nh, nw, row_degrees,
                                                       max_degree, sel_idx, sel_cnt, scores);
  CAST_CUDA_TRY(cudaGetLastError());
  return CAST_OK;
}

// ===========================================================================
// block-sparse attention
// ===========================================================================

// How the attention launch is cut into CTAs.  The kernel runs one CTA per
// work item (two 128-row query tiles of one (b*h, query block), or one
// single tile), heaviest first; the hardware hands CTAs to SMs in launch
// order, so the last wave leaves SMs idle while the longest items finish.
// The plan keeps the first items whole and cuts the items of the tail along
// their key tiles into parts whose partial results the kernel merges.  It is
// chosen by simulating that greedy dispatch over the SMs with the expected
// per-item work (count_hint, else max_degree key blocks per item): the
// threshold of tail work per SM below which items are cut, and the part
// length, are searched for the shortest simulated makespan.
struct AttnSplitPlan {
  int n_whole = 0, n_split = 0, n_parts = 0;
  int n_conv = 0;  // tail pairs run as two single tiles (no cut items then)
  std::vector<uint16_t> first, tiles;
  size_t ws_bytes = 0;
};

static size_t attn_counter_bytes(int n_split) { return ((size_t)n_split * 4 + 255) / 256 * 256; }

static AttnSplitPlan plan_attention_split(int BH, int nqb, int q_tiles, int k_tiles,
                                          int max_degree, const int32_t *count_hint, int n_sms,
                                          bool allow_cut) {
  using castk::kMaxItemParts;
  using castk::kMaxSplitItems;
  const int full_pairs = q_tiles / 2;
  const int n_full = BH * nqb * full_pairs;
  const int n_items = n_full + (q_tiles % 2 ? BH * nqb : 0);
  const int deg = std::min(max_degree, castk::kMaxBlockList);
  // key tiles (T) and cost per item, in the kernel's item order
  std::vector<int> T(n_items);
  std::vector<double> cost(n_items);
  for (int x = 0; x < n_items; ++x) {
    int bh, qb, unused;
    bool pair_item = x < n_full;
    if (pair_item)
      castk::item_coords(x, BH, nqb, full_pairs, bh, qb, unused);
    else
      castk::item_coords(x - n_full, BH, nqb, 1, bh, qb, unused);
    const int c = count_hint ? std::min(std::max(count_hint[(size_t)bh * nqb + qb], 0), deg) : deg;
    T[x] = c * k_tiles;
    // a single tile splits its key tiles over both softmax warpgroups
    cost[x] = pair_item || T[x] < 2 ? T[x] : 0.5 * T[x];
  }
  // Per-CTA cost in 128-key tile steps (launch, setup, pipeline fill and
  // drain, epilogue: ~9 us, ~4 tile steps, in CTA timelines on B200) and the
  // extra cost of a cut part (partial result written and merged: ~2.5).
  const double kCtaCost = 4.0, kPartCost = 2.5;
  auto simulate = [&](const std::vector<double> &d) {
    std::priority_queue<double, std::vector<double>, std::greater<double>> sm;
    for (int i = 0; i < n_sms; ++i) sm.push(0.0);
    double end = 0.0;
    for (double w : d) {
      const double t = sm.top() + w + kCtaCost;
      sm.pop();
      sm.push(t);
      end = std::max(end, t);
    }
    return end;
  };
  std::vector<double> suffix(n_items + 1, 0.0);
  for (int x = n_items - 1; x >= 0; --x) suffix[x] = suffix[x + 1] + cost[x];

  AttnSplitPlan best;
  best.n_whole = n_items;
  const double t_whole = simulate(cost);
  double best_t = t_whole;
  std::vector<double> d;
  // Converted pairs: the last n_conv pair items (the lightest pairs) run as
  // two single query tiles each, after the native single tiles; a single
  // tile shares its key tiles between both softmax warpgroups, so each half
  // costs half the pair.  Taken for a 2 % simulated gain.
  for (int n_conv = 4; n_conv <= n_full; n_conv += 4) {
    d.assign(cost.begin(), cost.begin() + (n_full - n_conv));
    d.insert(d.end(), cost.begin() + n_full, cost.end());
    for (int x = n_full - n_conv; x < n_full; ++x) d.insert(d.end(), 2, 0.5 * cost[x]);
    const double t = simulate(d);
    if (t < 0.98 * t_whole && t < best_t - 1e-9) {
      best_t = t;
      best.n_conv = n_conv;
    }
  }
  // Cut items: must beat running every item whole by 5 %, since the
  // simulation does not see every cost of the cut parts.
  std::vector<int> nparts;
  for (int thr = 4; allow_cut && thr <= 64; thr += 4) {
    int X = 0;
    while (X < n_items && suffix[X] > (double)thr * n_sms) ++X;
    if (X == n_items || n_items - X > kMaxSplitItems) continue;
    for (int len = 4; len <= 64; len += 4) {
      d.assign(cost.begin(), cost.begin() + X);
      nparts.assign(n_items - X, 1);
      int total = 0;
      for (int x = X; x < n_items; ++x) {
        const int n = std::max(1, std::min({(T[x] + len - 1) / len, kMaxItemParts, T[x]}));
        nparts[x - X] = n;
        total += n;
        for (int j = 0; j < n; ++j) d.push_back(cost[x] / n + (n > 1 ? kPartCost : 0.0));
      }
      if (total > 65535) continue;
      const double t = simulate(d);
      if (t < 0.95 * t_whole && t < best_t - 1e-9) {
        best_t = t;
        best.n_conv = 0;
        best.n_whole = X;
        best.n_split = n_items - X;
        best.n_parts = total;
        best.first.assign(1, 0);
        best.tiles.clear();
        for (int x = X; x < n_items; ++x) {
          best.first.push_back((uint16_t)(best.first.back() + nparts[x - X]));
          best.tiles.push_back((uint16_t)std::min(T[x], 65535));
        }
      }
    }
  }
  if (best.n_conv > 0) {  // the conversion won: no cut items
    best.n_whole = n_items;
    best.n_split = best.n_parts = 0;
    best.first.clear();
    best.tiles.clear();
  }
  if (best.n_split > 0)
    best.ws_bytes = attn_counter_bytes(best.n_split) +
                    (size_t)best.n_parts * castk::kPartSlotFloats * sizeof(float);
  return best;
}

// Plans are cached per (shape, hint, SM count): the search runs once per
// problem shape.
static std::mutex g_attn_plan_mutex;
static std::map<std::vector<int32_t>, AttnSplitPlan> g_attn_plans;

static AttnSplitPlan attention_plan(int BH, int nqb, int q_tiles, int k_tiles, int max_degree,
                                    const int32_t *count_hint, int n_sms, bool allow_cut) {
  std::vector<int32_t> key = {BH, nqb, q_tiles, k_tiles, max_degree, n_sms, count_hint ? 1 : 0,
                              allow_cut ? 1 : 0};
  if (count_hint) key.insert(key.end(), count_hint, count_hint + (size_t)BH * nqb);
  std::lock_guard<std::mutex> lock(g_attn_plan_mutex);
  auto it = g_attn_plans.find(key);
  if (it != g_attn_plans.end()) return it->second;
  if (g_attn_plans.size() >= 64) g_attn_plans.clear();
  AttnSplitPlan plan =
      plan_attention_split(BH, nqb, q_tiles, k_tiles, max_degree, count_hint, n_sms, allow_cut);
  g_attn_plans.emplace(std::move(key), plan);
  return plan;
}

static int attention_dims_ok(int B, int H, int Lq, int Lk, int q_block, int k_block, int max_degree) {
  if (B <= 0 || H <= 0 || Lq <= 0 || Lk <= 0 || q_block <= 0 || k_block <= 0 || max_degree <= 0)
    return fail(CAST_ERR_INVALID_ARGUMENT, "non-positive size");
  return CAST_OK;
}

extern "C" size_t cast_rcsa_attention_workspace_bytes(int B, int H, int Lq, int Lk, int q_block,
                                                       int k_block, int max_degree,
                                                       const int32_t *count_hint) {
  if (attention_dims_ok(B, H, Lq, Lk, q_block, k_block, max_degree)) return 0;
  int n_sms = 0;
  if (current_device_sm100(&n_sms)) return 0;
  return attention_plan(B * H, ceil_div(Lq, q_block), ceil_div(q_block, 128), ceil_div(k_block, 128),
                        max_degree, count_hint, n_sms, true)
      .ws_bytes;
}

// The fused all-gather of a head-sharded call (cast_rcsa_attention_peers).
struct PeerArgs {
  int n_peers = 0;
  const uint32_t *calls = nullptr;
  uint32_t *done_ticket = nullptr;
  void *const *peer_out = nullptr;
  uint32_t *const *peer_flag = nullptr;
};

static int attention_impl(const void *q, const void *k, const void *v, const int8_t *q_codes,
                          const float *q_scales, const int8_t *k_codes, const float *k_scales,
                          const uint8_t *qk_mode, const int32_t *indices, const int32_t *counts,
                          int max_degree, const uint8_t *key_valid, int B, int H, int Lq, int Lk,
                          int D, int q_block, int k_block, float sm_scale, void *out, float *lse,
                          const int32_t *count_hint, void *workspace, size_t workspace_bytes,
                          const PeerArgs &peers, cast_stream_t stream) {
  if (!q || !k || !v || !indices || !counts || !out)
    return fail(CAST_ERR_INVALID_ARGUMENT, "q, k, v, indices, counts and out are required");
  int st = attention_dims_ok(B, H, Lq, Lk, q_block, k_block, max_degree);
  if (st) return st;
  if (D != 128) return fail(CAST_ERR_UNSUPPORTED, "attention head_dim %d (supported: 128)", D);
  if (max_degree > castk::kMaxBlockList)
    return fail(CAST_ERR_UNSUPPORTED, "max_degree %d > %d key blocks per query block",
                max_degree, castk::kMaxBlockList);
  const bool have_codes = q_codes && k_codes && q_scales && k_scales;
  if ((q_codes || k_codes) && !have_codes)
    return fail(CAST_ERR_INVALID_ARGUMENT, "int8 QK^T needs q_codes, q_scales, k_codes and k_scales");
  if (qk_mode && !have_codes)
    return fail(CAST_ERR_INVALID_ARGUMENT, "qk_mode given without int8 codes");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) ||
      (q_codes && !aligned16(q_codes)) || (k_codes && !aligned16(k_codes)) ||
      (key_valid && !aligned16(key_valid)) || (workspace && !aligned16(workspace)))
    return fail(CAST_ERR_ALIGNMENT, "tensor base pointers must be 16-byte aligned");
  if (!(sm_scale > 0.0f) || !std::isfinite(sm_scale))
    return fail(CAST_ERR_INVALID_ARGUMENT, "sm_scale must be positive and finite");
  if ((long long)B * H * std::max(Lq, Lk) >= (1ll << 31))
    return fail(CAST_ERR_UNSUPPORTED, "B*H*L exceeds the 32-bit TMA coordinate range");
  int n_sms = 0;
  st = current_device_sm100(&n_sms);
  if (st) return st;

  const int BH = B * H;
  CUtensorMap tm_q8, tm_k8, tm_q16, tm_k16, tm_v, tm_vb;
  memset(&tm_q8, 0, sizeof(tm_q8));
  memset(&tm_k8, 0, sizeof(tm_k8));
  // Values of whole key blocks through a block-structured map [BH][block][row]
  // [D]: the rows a block's last 128-row tile reads past the block's end are
  // outside the map and arrive as zeros, so whatever the next block holds
  // (it may be unselected, even non-finite) never meets the zero
  // probabilities of those masked rows.  The ragged last block (Lk not a
  // multiple of the block) and blocks shorter than a tile use the plain map,
  // whose rows past Lk are zeros too.
  const int nkb_full = k_block >= 128 ? Lk / k_block : 0;
  if (nkb_full > 0) {
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)k_block, (uint64_t)nkb_full, (uint64_t)BH};
    const uint64_t strides[3] = {(uint64_t)D * 2, (uint64_t)k_block * D * 2, (uint64_t)Lk * D * 2};
    if ((st = make_map_4d_strided(&tm_vb, v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, dims, strides, 64, 128,
                                  CU_TENSOR_MAP_SWIZZLE_128B)))
      return st;
  }
  if ((st = make_map_3d(&tm_q16, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, D, Lq, BH, 64, 128,
                        CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if ((st = make_map_3d(&tm_k16, k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, D, Lk, BH, 64, 128,
                        CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if ((st = make_map_3d(&tm_v, v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, D, Lk, BH, 64, 128,
                        CU_TENSOR_MAP_SWIZZLE_128B)))
    return st;
  if (nkb_full == 0) tm_vb = tm_v;  // never read
  if (have_codes) {
    if ((st = make_map_3d(&tm_q8, q_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, D, Lq, BH, 128, 128,
                          CU_TENSOR_MAP_SWIZZLE_128B)))
      return st;
    if ((st = make_map_3d(&tm_k8, k_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, D, Lk, BH, 128, 128,
                          CU_TENSOR_MAP_SWIZZLE_128B)))
      return st;
  } else {
    tm_q8 = tm_q16;  // never read: every work item runs bf16
    tm_k8 = tm_k16;
  }

  castk::AttnParams p;
  p.indices = indices;
  p.counts = counts;
  p.q_scales = q_scales;
  p.k_scales = k_scales;
  p.qk_mode = qk_mode;
  p.key_valid = key_valid;
  p.out = static_cast<__nv_bfloat16 *>(out);
  p.lse = lse;
  p.max_degree = max_degree;
  p.BH = BH;
  p.Lq = Lq;
  p.Lk = Lk;
  p.q_block = q_block;
  p.k_block = k_block;
  p.nqb = ceil_div(Lq, q_block);
  p.nkb = ceil_div(Lk, k_block);
  p.nkb_full = nkb_full;
  p.q_tiles = ceil_div(q_block, 128);
  p.k_tiles = ceil_div(k_block, 128);
  p.full_pairs = p.q_tiles / 2;
  p.n_full_items = BH * p.nqb * p.full_pairs;
  p.default_mode = have_codes ? 1 : 0;
  p.sm_scale_log2 = sm_scale * 1.4426950408889634f;
  const int n_items = p.n_full_items + (p.q_tiles % 2 ? BH * p.nqb : 0);
  p.n_items = n_items;
  p.n_whole = n_items;
  p.n_split = 0;
  p.part_counter = nullptr;
  p.part_ws = nullptr;
  memset(p.part_first, 0, sizeof(p.part_first));
  memset(p.part_tiles, 0, sizeof(p.part_tiles));
  p.n_peers = peers.n_peers;
  p.calls = peers.calls;
  p.done_ticket = peers.done_ticket;
  for (int r = 0; r < castk::kMaxPeers; ++r) {
    p.peer_out[r] = r < peers.n_peers ? static_cast<__nv_bfloat16 *>(peers.peer_out[r]) : nullptr;
    p.peer_flag[r] = r < peers.n_peers ? peers.peer_flag[r] : nullptr;
  }
  // Items are cut only with a workspace; converting tail pairs needs none.
  const AttnSplitPlan plan = attention_plan(BH, p.nqb, p.q_tiles, p.k_tiles, max_degree, count_hint,
                                            n_sms, workspace != nullptr);
  p.n_conv = plan.n_conv;
  int grid = n_items + plan.n_conv;
  if (workspace) {
    if (workspace_bytes < plan.ws_bytes)
      return fail(CAST_ERR_WORKSPACE, "workspace of %zu bytes < %zu required", workspace_bytes,
                  plan.ws_bytes);
    if (plan.n_split > 0) {
      p.n_whole = plan.n_whole;
      p.n_split = plan.n_split;
      p.part_counter = static_cast<int *>(workspace);
      p.part_ws = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) +
                                            attn_counter_bytes(plan.n_split));
      std::copy(plan.first.begin(), plan.first.end(), p.part_first);
      std::copy(plan.tiles.begin(), plan.tiles.end(), p.part_tiles);
      grid = plan.n_whole + plan.n_parts;
    }
  }

  static std::once_flag attr_once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(attr_once, [] {
    attr_err = cudaFuncSetAttribute(castk::rcsa_attention_kernel,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    castk::AttnSmem::alloc);
  });
  CAST_CUDA_TRY(attr_err);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  castk::rcsa_attention_kernel<<<grid, castk::kAttnThreads, castk::AttnSmem::alloc, s>>>(
      tm_q8, tm_k8, tm_q16, tm_k16, tm_v, tm_vb, p);
  CAST_CUDA_TRY(cudaGetLastError());
  return CAST_OK;
}

extern "C" int cast_rcsa_attention(const void *q, const void *k, const void *v,
                                   const int8_t *q_codes, const float *q_scales,
                                   const int8_t *k_codes, const float *k_scales,
                                   const uint8_t *qk_mode, const int32_t *indices,
                                   const int32_t *counts, int max_degree,
                                   const uint8_t *key_valid, int B, int H, int Lq, int Lk, int D,
                                   int q_block, int k_block, float sm_scale, void *out,
                                   float *lse, const int32_t *count_hint, void *workspace,
                                   size_t workspace_bytes, cast_stream_t stream) {
  return attention_impl(q, k, v, q_codes, q_scales, k_codes, k_scales, qk_mode, indices, counts,
                        max_degree, key_valid, B, H, Lq, Lk, D, q_block, k_block, sm_scale, out, lse,
                        count_hint, workspace, workspace_bytes, PeerArgs{}, stream);
}

extern "C" int cast_rcsa_attention_peers(
    const void *q, const void *k, const void *v, const int8_t *q_codes, const float *q_scales,
    const int8_t *k_codes, const float *k_scales, const uint8_t *qk_mode, const int32_t *indices,
    const int32_t *counts, int max_degree, const uint8_t *key_valid, int B, int H, int Lq, int Lk,
    int D, int q_block, int k_block, float sm_scale, void *out, float *lse,
    const int32_t *count_hint, void *workspace, size_t workspace_bytes, int n_peers,
    void *const *peer_out, uint32_t *const *peer_flag, uint32_t *done_ticket,
    const uint32_t *calls, cast_stream_t stream) {
  if (n_peers < 0 || n_peers > castk::kMaxPeers)
    return fail(CAST_ERR_UNSUPPORTED, "%d peers (at most %d)", n_peers, castk::kMaxPeers);
  if (n_peers > 0) {
    if (!peer_out || !peer_flag || !done_ticket || !calls)
      return fail(CAST_ERR_INVALID_ARGUMENT, "peer_out, peer_flag, done_ticket and calls are required");
    for (int r = 0; r < n_peers; ++r)
      if (!peer_out[r] || !peer_flag[r] || !aligned16(peer_out[r]) || (reinterpret_cast<uintptr_t>(peer_flag[r]) & 3))
        return fail(CAST_ERR_ALIGNMENT, "peer %d: output must be 16-byte and its flag 4-byte aligned", r);
  }
  PeerArgs peers;
  peers.n_peers = n_peers;
  peers.calls = calls;
  peers.done_ticket = done_ticket;
  peers.peer_out = peer_out;
  peers.peer_flag = peer_flag;
  return attention_impl(q, k, v, q_codes, q_scales, k_codes, k_scales, qk_mode, indices, counts,
                        max_degree, key_valid, B, H, Lq, Lk, D, q_block, k_block, sm_scale, out, lse,
                        count_hint, workspace, workspace_bytes, peers, stream);
}

// ===========================================================================
// peer buffers (CUDA IPC, no multicast) and the gather's completion wait
// ===========================================================================
namespace castk {
// One thread per source rank: until the rank's flag holds this call's number
// (*calls + 1; acquire, system scope), bounded by kWaitLimitNs -- a wait that
// gives up sets the device error word; then the call counter advances.
__global__ void peer_wait_kernel(const uint32_t *flags, int n_src, int self_rank, uint32_t *calls) {
  const int r = threadIdx.x;
  const uint32_t call = *calls + 1u;
  if (r < n_src && r != self_rank && castdev::ld_acquire_sys(flags + r) != call) {
    const uint64_t t0 = castdev::global_timer_ns();
    for (uint32_t spin = 0;; ++spin) {
      if (castdev::ld_acquire_sys(flags + r) == call) break;
      if ((spin & 255u) == 255u && castdev::global_timer_ns() - t0 > castdev::kWaitLimitNs) {
        atomicExch(&g_cast_device_error, (int)CAST_ERR_DEVICE_TIMEOUT);
        break;
      }
    }
  }
  __syncwarp();
  if (r == 0) *calls = call;
}
}  // namespace castk

namespace castk {
struct PeerPushArgs {
  int n_peers;
  uint32_t *done_ticket;
  const uint32_t *calls;
  uint4 *dst[kMaxPeers];
  uint32_t *flag[kMaxPeers];
};

// The gather as its own launch after the attention: every CTA streams a share
// of this rank's output slot (16-byte loads, coalesced) into the same offset
// of every peer's gathered buffer, fences its stores at system scope and takes
// a ticket; the last CTA raises this rank's flag in every peer to the call's
// number (*calls + 1) and resets the ticket.
__global__ void __launch_bounds__(512) peer_push_kernel(const uint4 *__restrict__ src, size_t n16,
                                                        PeerPushArgs a) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < n16; i += 4 * stride) {
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = __ldcs(src + i + u * stride);
    for (int r = 0; r < a.n_peers; ++r)
#pragma unroll
      for (int u = 0; u < 4; ++u) a.dst[r][i + u * stride] = v[u];
  }
  for (; i < n16; i += stride) {
    const uint4 v = __ldcs(src + i);
    for (int r = 0; r < a.n_peers; ++r) a.dst[r][i] = v;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t t = atomicAdd(a.done_ticket, 1u);
    if (t == gridDim.x - 1) {
      __threadfence_system();
      const uint32_t call = *reinterpret_cast<const volatile uint32_t *>(a.calls) + 1u;
      for (int r = 0; r < a.n_peers; ++r) castdev::st_release_sys(a.flag[r], call);
      atomicExch(a.done_ticket, 0u);
    }
  }
}
}  // namespace castk

extern "C" int cast_peer_push(const void *src, size_t bytes, int n_peers, void *const *peer_dst,
                              uint32_t *const *peer_flag, uint32_t *done_ticket, const uint32_t *calls,
                              cast_stream_t stream) {
  if (!src || !bytes || (bytes & 15) || !aligned16(src))
    return fail(CAST_ERR_ALIGNMENT, "src must be 16-byte aligned, bytes a positive multiple of 16");
  if (n_peers < 1 || n_peers > castk::kMaxPeers)
    return fail(CAST_ERR_UNSUPPORTED, "%d peers (1..%d)", n_peers, castk::kMaxPeers);
  if (!peer_dst || !peer_flag || !done_ticket || !calls)
    return fail(CAST_ERR_INVALID_ARGUMENT, "peer_dst, peer_flag, done_ticket and calls are required");
  castk::PeerPushArgs a;
  memset(&a, 0, sizeof(a));
  a.n_peers = n_peers;
  a.done_ticket = done_ticket;
  a.calls = calls;
  for (int r = 0; r < n_peers; ++r) {
    if (!peer_dst[r] || !peer_flag[r] || !aligned16(peer_dst[r]) || (reinterpret_cast<uintptr_t>(peer_flag[r]) & 3))
      return fail(CAST_ERR_ALIGNMENT, "peer %d: destination must be 16-byte and its flag 4-byte aligned", r);
    a.dst[r] = static_cast<uint4 *>(peer_dst[r]);
    a.flag[r] = peer_flag[r];
  }
  int n_sms = 0;
  int st = current_device_sm100(&n_sms);
  if (st) return st;
  castk::peer_push_kernel<<<n_sms, 512, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4 *>(src), bytes / 16, a);
  CAST_CUDA_TRY(cudaGetLastError());
  return CAST_OK;
}

namespace castk {
// After a copy engine has moved this rank's slot into a peer's buffer (the
// copy precedes this launch in its stream): one thread raises this rank's
// flag in that peer to the call's number.
__global__ void peer_signal_kernel(uint32_t *peer_flag, const uint32_t *calls) {
  __threadfence_system();
  castdev::st_release_sys(peer_flag, *reinterpret_cast<const volatile uint32_t *>(calls) + 1u);
}
}  // namespace castk

extern "C" int cast_peer_send(void *peer_dst, const void *src, size_t bytes, uint32_t *peer_flag,
                              const uint32_t *calls, cast_stream_t stream) {
  if (!peer_dst || !src || !bytes || !peer_flag || !calls)
    return fail(CAST_ERR_INVALID_ARGUMENT, "peer_dst, src, bytes, peer_flag and calls are required");
  if (reinterpret_cast<uintptr_t>(peer_flag) & 3) return fail(CAST_ERR_ALIGNMENT, "peer_flag must be 4-byte aligned");
  int st = current_device_sm100(nullptr);
  if (st) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  CAST_CUDA_TRY(cudaMemcpyAsync(peer_dst, src, bytes, cudaMemcpyDeviceToDevice, s));
  castk::peer_signal_kernel<<<1, 1, 0, s>>>(peer_flag, calls);
  CAST_CUDA_TRY(cudaGetLastError());
  return CAST_OK;
}

extern "C" int cast_peer_alloc(size_t bytes, void **ptr, void *ipc_handle) {
  if (!ptr || !ipc_handle || bytes == 0) return fail(CAST_ERR_INVALID_ARGUMENT, "bytes, ptr and handle required");
  int st = current_device_sm100(nullptr);
  if (st) return st;
  void *p = nullptr;
  CAST_CUDA_TRY(cudaMalloc(&p, bytes));
  cudaError_t e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t *>(ipc_handle), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(CAST_ERR_CUDA, "peer buffer: %s", cudaGetErrorString(e));
  }
  *ptr = p;
  return CAST_OK;
}

extern "C" int cast_peer_open(const void *ipc_handle, void **ptr) {
  if (!ptr || !ipc_handle) return fail(CAST_ERR_INVALID_ARGUMENT, "handle and ptr required");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  CAST_CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return CAST_OK;
}

extern "C" int cast_peer_close(void *ptr) {
  if (!ptr) return fail(CAST_ERR_INVALID_ARGUMENT, "ptr required");
  CAST_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
  return CAST_OK;
}

extern "C" int cast_peer_free(void *ptr) {
  if (!ptr) return fail(CAST_ERR_INVALID_ARGUMENT, "ptr required");
  CAST_CUDA_TRY(cudaFree(ptr));
  return CAST_OK;
}

extern "C" int cast_peer_wait(const uint32_t *flags, int n_src, int self_rank, uint32_t *calls,
                              cast_stream_t stream) {
  if (!flags || !calls || n_src <= 0 || n_src > castk::kMaxPeers + 1 || self_rank < 0 ||
      self_rank >= n_src)
    return fail(CAST_ERR_INVALID_ARGUMENT, "flags, calls, %d sources (1..%d), rank %d", n_src,
                castk::kMaxPeers + 1, self_rank);
  int st = current_device_sm100(nullptr);
  if (st) return st;
  castk::peer_wait_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(flags, n_src, self_rank,
                                                                                  calls);
  CAST_CUDA_TRY(cudaGetLastError());
  return CAST_OK;
}

// ===========================================================================
// compact-layout packing (+ RoPE phase) and the output scatter
// ===========================================================================
static int grid_rows(long long rows, int n_sms) {
  // enough CTAs of 128 threads to fill every SM several times over
  return (int)std::min<long long>(rows, (long long)n_sms * 16);
}

extern "C" int cast_compact_pack(const void *q, const void *k, const void *v, int in_dtype,
                                 const float *phase, int phase_heads, const int32_t *block_indices,
                                 int B, int L, int H, int D, int P, void *q_out, void *k_out,
                                 void *v_out, cast_stream_t stream) {
  if (!q || !k || !v || !block_indices || !q_out || !k_out || !v_out)
    return fail(CAST_ERR_INVALID_ARGUMENT, "q, k, v, block_indices and the outputs are required");
  if (B <= 0 || L <= 0 || H <= 0 || P <= 0) return fail(CAST_ERR_INVALID_ARGUMENT, "non-positive size");
  if (D != castk::kCompactD) return fail(CAST_ERR_UNSUPPORTED, "compact path head_dim %d (supported: 128)", D);
  if (in_dtype != 0 && in_dtype != 1)
    return fail(CAST_ERR_INVALID_ARGUMENT, "in_dtype %d (0 = bf16, 1 = fp32)", in_dtype);
  if (phase && phase_heads != 1 && phase_heads != H)
    return fail(CAST_ERR_INVALID_ARGUMENT, "phase_heads %d must be 1 or H = %d", phase_heads, H);
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(q_out) || !aligned16(k_out) ||
      !aligned16(v_out) || (phase && !aligned16(phase)))
    return fail(CAST_ERR_ALIGNMENT, "tensor base pointers must be 16-byte aligned");
  int n_sms = 0;
  int st = current_device_sm100(&n_sms);
  if (st) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int grid = grid_rows((long long)B * P, n_sms);
  const float2 *ph = reinterpret_cast<const float2 *>(phase);
  auto *qo = static_cast<__nv_bfloat16 *>(q_out);
  auto *ko = static_cast<__nv_bfloat16 *>(k_out);
  auto *vo = static_cast<__nv_bfloat16 *>(v_out);
  if (in_dtype == 0)
    castk::compact_pack_kernel<__nv_bfloat16><<<grid, castk::kCompactThreads, 0, s>>>(
        static_cast<const __nv_bfloat16 *>(q), static_cast<const __nv_bfloat16 *>(k),
        static_cast<const __nv_bfloat16 *>(v), ph, phase_heads, block_indices, B, L, H, P, qo, ko, vo);
  else
    castk::compact_pack_kernel<float><<<grid, castk::kCompactThreads, 0, s>>>(
        static_cast<const float *>(q), static_cast<const float *>(k), static_cast<const float *>(v), ph,
        phase_heads, block_indices, B, L, H, P, qo, ko, vo);
  CAST_CUDA_TRY(cudaGetLastError());
  return CAST_OK;
}

extern "C" int cast_compact_unpack(const void *packed, const int32_t *token_to_packed, int B, int L,
                                   int H, int D, int P, void *out, cast_stream_t stream) {
  if (!packed || !token_to_packed || !out)
    return fail(CAST_ERR_INVALID_ARGUMENT, "packed, token_to_packed and out are required");
  if (B <= 0 || L <= 0 || H <= 0 || P <= 0) return fail(CAST_ERR_INVALID_ARGUMENT, "non-positive size");
  if (D != castk::kCompactD) return fail(CAST_ERR_UNSUPPORTED, "compact path head_dim %d (supported: 128)", D);
  if (!aligned16(packed) || !aligned16(out))
    return fail(CAST_ERR_ALIGNMENT, "tensor base pointers must be 16-byte aligned");
  int n_sms = 0;
  int st = current_device_sm100(&n_sms);
  if (st) return st;
  castk::compact_unpack_kernel<<<grid_rows((long long)B * L, n_sms), castk::kCompactThreads, 0,
                                 reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16 *>(packed), token_to_packed, B, L, H, P,
      static_cast<__nv_bfloat16 *>(out));
  CAST_CUDA_TRY(cudaGetLastError());
  return CAST_OK;
}

// ===========================================================================
// control-barycentric two-anchor writer
// ===========================================================================
extern "C" int cast_barycentric_pair_write(const float *active_residual, const float *weights,
                                           const int32_t *source_pairs, const int32_t *target_frames,
                                           float *output, int A, int T, int N, long long spatial_channels,
                                           int arithmetic_mode, cast_stream_t stream) {
  if (!active_residual || !weights || !source_pairs || !target_frames || !output)
    return fail(CAST_ERR_INVALID_ARGUMENT, "all tensors are required");
  if (A <= 0 || T <= 0 || N <= 0 || spatial_channels <= 0)
    return fail(CAST_ERR_INVALID_ARGUMENT, "non-positive size");
  if (arithmetic_mode < 0 || arithmetic_mode > 3)
    return fail(CAST_ERR_INVALID_ARGUMENT, "arithmetic_mode %d (0..3)", arithmetic_mode);
  if (!aligned16(active_residual) || !aligned16(output))
    return fail(CAST_ERR_ALIGNMENT, "tensor base pointers must be 16-byte aligned");
  int n_sms = 0;
  int st = current_device_sm100(&n_sms);
  if (st) return st;
  const long long vec = (spatial_channels & 3) == 0 ? spatial_channels / 4 : spatial_channels;
  // 4 CTAs per SM, grid-strided over the frame (every CTA walks all rows)
  const int grid = (int)std::min<long long>((long long)n_sms * 4,
                                            (vec + castk::kBaryThreads - 1) / castk::kBaryThreads);
  castk::barycentric_pair_kernel<<<grid, castk::kBaryThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      active_residual, weights, source_pairs, target_frames, output, spatial_channels, A, T, N,
      arithmetic_mode == 0 ? 2 : arithmetic_mode);
  CAST_CUDA_TRY(cudaGetLastError());
  return CAST_OK;
}

extern "C" int cast_barycentric_weights(const void *plucker, int plucker_bf16, int B, int rows, int P,
                                        int S, int T, int M, const float *mouse, int mouse_len,
                                        int mouse_ch, const float *keyboard, int keyboard_len,
                                        int keyboard_ch, const float *mouse_memory,
                                        int mouse_memory_len, int mouse_memory_ch,
                                        const float *keyboard_memory, int keyboard_memory_len,
                                        int keyboard_memory_ch, int n_targets,
                                        const int32_t *targets, const float *prior, float lambda_p,
                                        float lambda_a, float *weights, const int32_t *slots,
                                        int32_t *source_pairs, int32_t *target_frames,
                                        cast_stream_t stream) {
  using castk::kLiftMaxAct;
  using castk::kLiftMaxFeat;
  using castk::kLiftMaxTargets;
  if (!plucker || !targets || !prior || !weights)
    return fail(CAST_ERR_INVALID_ARGUMENT, "plucker, targets, prior and weights are required");
  if (B <= 0 || P <= 0 || P > kLiftMaxFeat || S <= 0 || T <= 0 || M < 0 || M >= T ||
      rows < T * S || n_targets <= 0 || n_targets > kLiftMaxTargets)
    return fail(CAST_ERR_INVALID_ARGUMENT,
                "bad sizes (B=%d rows=%d P=%d S=%d T=%d memory=%d targets=%d; P <= %d, targets <= %d)",
                B, rows, P, S, T, M, n_targets, kLiftMaxFeat, kLiftMaxTargets);
  const int cm = mouse ? mouse_ch : 0, ck = keyboard ? keyboard_ch : 0;
  const int mm = mouse_memory ? mouse_memory_ch : 0, km = keyboard_memory ? keyboard_memory_ch : 0;
  if (cm + ck > kLiftMaxAct) return fail(CAST_ERR_UNSUPPORTED, "more than %d control channels", kLiftMaxAct);
  if ((mouse && (mouse_len <= 0 || mouse_ch <= 0)) || (keyboard && (keyboard_len <= 0 || keyboard_ch <= 0)) ||
      (mouse_memory && (mouse_memory_len <= 0 || mouse_memory_ch <= 0)) ||
      (keyboard_memory && (keyboard_memory_len <= 0 || keyboard_memory_ch <= 0)))
    return fail(CAST_ERR_INVALID_ARGUMENT, "control sequences must be non-empty");
  if ((mouse_memory || keyboard_memory) && (!(mouse || keyboard) || M == 0 || mm + km != cm + ck))
    return fail(CAST_ERR_INVALID_ARGUMENT,
                "Memory/Current action dimensions disagree (memory %d, current %d channels, memory frames %d)",
                mm + km, cm + ck, M);
  castk::LiftParams p;
  memset(&p, 0, sizeof(p));
  for (int n = 0; n < n_targets; ++n) {
    for (int j = 0; j < 3; ++j) {
      const int f = targets[3 * n + j];
      if (f < 0 || f >= T) return fail(CAST_ERR_INVALID_ARGUMENT, "target %d frame %d outside [0,%d)", n, f, T);
      p.targets[n][j] = f;
    }
    p.prior[n][0] = prior[2 * n];
    p.prior[n][1] = prior[2 * n + 1];
    if (slots) {
      p.slots[n][0] = slots[2 * n];
      p.slots[n][1] = slots[2 * n + 1];
    }
  }
  if ((slots != nullptr) != (source_pairs != nullptr) || (source_pairs != nullptr) != (target_frames != nullptr))
    return fail(CAST_ERR_INVALID_ARGUMENT, "slots, source_pairs and target_frames go together");
  p.pairs_out = source_pairs;
  p.frames_out = target_frames;
  int st = current_device_sm100(nullptr);
  if (st) return st;
  p.plucker = plucker, p.plucker_bf16 = plucker_bf16 ? 1 : 0, p.P = P, p.S = S, p.T = T, p.M = M;
  p.rows = rows;
  p.cur[0] = castk::LiftCond{mouse, mouse_len, mouse_ch};
  p.cur[1] = castk::LiftCond{keyboard, keyboard_len, keyboard_ch};
  p.mem[0] = castk::LiftCond{mouse_memory, mouse_memory_len, mm};
  p.mem[1] = castk::LiftCond{keyboard_memory, keyboard_memory_len, km};
  p.action = (mouse || keyboard) ? 1 : 0;
  p.lp = lambda_p, p.la = lambda_a, p.weights = weights, p.N = n_targets;
  castk::barycentric_weights_kernel<<<dim3(n_targets, B), castk::kLiftThreads, 0,
                                       reinterpret_cast<cudaStream_t>(stream)>>>(p);
  CAST_CUDA_TRY(cudaGetLastError());
  return CAST_OK;
}

// ===========================================================================
// FC-PASM swap router
// ===========================================================================
struct SwapLayout {
  size_t cand, proxy, err, limit, best, obj, ctl, total;
};

static bool swap_shape(int B, int H, int Q, int K, int D, int S, int M, int mult, int historical,
                       int same_bank, int G, castk::SwapShape *p) {
  if (B <= 0 || H <= 0 || Q <= 0 || K <= 0 || D <= 0 || S <= 0 || M < 0 || M >= Q || mult < 1 ||
      G < 2 || (G & 1) || D % G)
    return false;
  p->B = B, p->H = H, p->Q = Q, p->K = K, p->D = D, p->S = S, p->M = M, p->R = Q - M, p->G = G;
  p->cand_blocks = historical ? M : K;
  p->Lc = (int)std::min<long long>(p->cand_blocks, (long long)mult * S);
  p->mult = mult, p->historical = historical ? 1 : 0, p->same_bank = same_bank ? 1 : 0;
  p->stage_v = 0;
  return p->cand_blocks > 0;
}

static SwapLayout swap_layout(const castk::SwapShape &p) {
  const size_t rows = (size_t)p.B * p.H * p.R, bh = (size_t)p.B * p.H;
  SwapLayout l;
  l.cand = 0;
  l.proxy = l.cand + align_up(rows * p.Lc * sizeof(int), 256);
  l.err = l.proxy + align_up(rows * p.Lc * p.G * sizeof(float), 256);
  l.limit = l.err + align_up(rows * p.G * sizeof(float), 256);
  l.best = l.limit + align_up(rows * sizeof(int), 256);
  l.obj = l.best + align_up(rows * sizeof(castk::SwapBest), 256);
  l.ctl = l.obj + align_up(2 * rows * sizeof(double), 256);
  l.total = l.ctl + 256;
  return l;
}

extern "C" size_t cast_swap_route_workspace_bytes(int B, int H, int Q, int K, int D, int S,
                                                  int memory_blocks, int candidate_multiplier,
                                                  int historical_only, int sketch_groups) {
  castk::SwapShape p;
  if (!swap_shape(B, H, Q, K, D, S, memory_blocks, candidate_multiplier, historical_only, 0,
                  sketch_groups, &p))
    return 0;
  return swap_layout(p).total;
}

extern "C" int cast_swap_objective(int n, int tiles, int bins, const float *u_re, const float *u_im,
                                   const float *v_re, const float *v_im, int cells,
                                   const float *cell_anchor_count, int n_targets,
                                   const float *const *target_theta,
                                   const float *const *target_affinity, const double *target_alpha,
                                   const int32_t *target_cells, int n_pairs,
                                   const float *const *pair_mean, const float *pair_mean_value,
                                   const int32_t *pair_cells, const int32_t *pair_matching,
                                   int require_fc_transport, float min_transport_affinity,
                                   float min_pair_transport_affinity, float lambda_anchor,
                                   float lambda_reconstruction, float *coefficient, float *hessian,
                                   uint8_t *row_gate, int32_t *gate, double *stats, float *operators,
                                   cast_stream_t stream) {
  using castk::kSwapObjMaxBins;
  using castk::kSwapObjMaxCells;
  using castk::kSwapObjMaxPairs;
  using castk::kSwapObjMaxTargets;
  if (!cell_anchor_count || !coefficient || !hessian || !gate || !stats || !operators)
    return fail(CAST_ERR_INVALID_ARGUMENT, "cell counts, coefficient, hessian, gate, stats and "
                                           "operators are required");
  if (n <= 0 || cells <= 0 || cells > kSwapObjMaxCells || n_targets <= 0 ||
      n_targets > kSwapObjMaxTargets || n_pairs < 0 || n_pairs > kSwapObjMaxPairs)
    return fail(CAST_ERR_UNSUPPORTED, "objective sizes (n=%d cells=%d targets=%d pairs=%d; at most "
                                      "%d cells, %d targets, %d pairs)", n, cells, n_targets, n_pairs,
                kSwapObjMaxCells, kSwapObjMaxTargets, kSwapObjMaxPairs);
  if ((long long)cells * n > 4096) return fail(CAST_ERR_UNSUPPORTED, "more than 4096 current rows");
  if (n_targets && (!target_theta || !target_affinity || !target_alpha || !target_cells))
    return fail(CAST_ERR_INVALID_ARGUMENT, "target tables are required");
  if (n_pairs && (!pair_mean || !pair_mean_value || !pair_cells || !pair_matching))
    return fail(CAST_ERR_INVALID_ARGUMENT, "pair tables are required");
  if (min_pair_transport_affinity > 0.f && !row_gate)
    return fail(CAST_ERR_INVALID_ARGUMENT, "the pair gate needs row_gate");
  castk::SwapObjParams p;
  memset(&p, 0, sizeof(p));
  bool sketched = false;
  for (int t = 0; t < n_targets; ++t) {
    const int lc = target_cells[2 * t], rc = target_cells[2 * t + 1];
    if (lc < 0 || lc >= cells || rc < 0 || rc >= cells)
      return fail(CAST_ERR_INVALID_ARGUMENT, "target %d cells (%d, %d) outside [0,%d)", t, lc, rc, cells);
    if ((target_theta[t] == nullptr) != (target_affinity[t] == nullptr))
      return fail(CAST_ERR_INVALID_ARGUMENT, "target %d: theta and affinity go together", t);
    const double a = target_alpha[t];
    p.t[t] = castk::SwapObjTarget{target_theta[t], target_affinity[t], (float)a, (float)(-(1.0 - a)),
                                  (float)(1.0 - a), (float)a, lc, rc};
    sketched |= target_theta[t] != nullptr;
  }
  if (sketched) {
    if (!u_re || !u_im || !v_re || !v_im || tiles <= 0 || bins <= 0 || tiles * bins > kSwapObjMaxBins)
      return fail(CAST_ERR_INVALID_ARGUMENT, "sketched targets need the transport basis "
                                             "(tiles x bins <= %d)", kSwapObjMaxBins);
  }
  for (int i = 0; i < n_pairs; ++i) {
    const int lo = pair_cells[2 * i], hi = pair_cells[2 * i + 1];
    if (lo < 0 || hi < lo || hi >= cells)
      return fail(CAST_ERR_INVALID_ARGUMENT, "pair %d cells [%d, %d] outside [0,%d)", i, lo, hi, cells);
    p.pr[i] = castk::SwapObjPair{pair_mean[i], pair_mean_value[i], lo, hi, pair_matching[i] ? 1 : 0};
  }
  int st = current_device_sm100(nullptr);
  if (st) return st;
  p.n = n, p.tiles = tiles, p.bins = bins, p.cells = cells, p.R = cells * n, p.T = n_targets;
  p.n_pairs = n_pairs;
  p.u_re = u_re, p.u_im = u_im, p.v_re = v_re, p.v_im = v_im;
  p.lam_a = lambda_anchor, p.lam_r = lambda_reconstruction;
  p.min_match = min_transport_affinity, p.min_pair = min_pair_transport_affinity;
  p.require_fc = require_fc_transport ? 1 : 0;
  p.pair_gate = min_pair_transport_affinity > 0.f ? 1 : 0;
  for (int c = 0; c < cells; ++c) p.cell_count[c] = cell_anchor_count[c];
  p.ops = operators, p.coef = coefficient, p.hess = hessian, p.row_gate = row_gate;
  p.gate = gate, p.stats = stats;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const dim3 g1(2 * n_targets, ceil_div(n * n, castk::kSwapObjThreads / 32));
  castk::swap_operator_kernel<<<g1, castk::kSwapObjThreads, 0, s>>>(p);
  CAST_CUDA_TRY(cudaGetLastError());
  const int g2 = std::max(1, std::min(1024, ceil_div(p.R * p.R + p.R, castk::kSwapObjThreads)));
  castk::swap_hessian_kernel<<<g2, castk::kSwapObjThreads, 0, s>>>(p);
  CAST_CUDA_TRY(cudaGetLastError());
  return CAST_OK;
}

extern "C" int cast_swap_route(const float *score, const float *pooled_value, long long *selected,
                               const long long *counts, const uint8_t *local, const uint8_t *row_gate,
                               const int32_t *gate, const float *coefficient, const float *hessian,
                               int B, int H, int Q,
                               int K, int D, int S, int memory_blocks, int candidate_multiplier,
                               int num_swap_rounds, float swap_eps, int sketch_groups,
                               int max_swaps_per_call, int historical_only, int same_bank_only,
                               double *stats, void *workspace, size_t workspace_bytes,
                               cast_stream_t stream) {
  if (!score || !pooled_value || !selected || !counts || !local || !coefficient || !hessian || !stats)
    return fail(CAST_ERR_INVALID_ARGUMENT, "score, pooled_value, selected, counts, local, "
                                           "coefficient, hessian and stats are required");
  castk::SwapShape p;
  if (!swap_shape(B, H, Q, K, D, S, memory_blocks, candidate_multiplier, historical_only,
                  same_bank_only, sketch_groups, &p))
    return fail(CAST_ERR_INVALID_ARGUMENT,
                "invalid shape (B=%d H=%d Q=%d K=%d D=%d S=%d memory_blocks=%d multiplier=%d "
                "sketch_groups=%d historical_only=%d)",
                B, H, Q, K, D, S, memory_blocks, candidate_multiplier, sketch_groups, historical_only);
  if (num_swap_rounds < 0 || num_swap_rounds > 2)
    return fail(CAST_ERR_INVALID_ARGUMENT, "num_swap_rounds %d (0..2)", num_swap_rounds);
  if (max_swaps_per_call < 0) return fail(CAST_ERR_INVALID_ARGUMENT, "negative max_swaps_per_call");
  if (!(swap_eps >= 0.f) || std::isinf(swap_eps))
    return fail(CAST_ERR_INVALID_ARGUMENT, "swap_eps must be finite and non-negative");
  size_t sm1 = (size_t)(2 * K + D + 32 + p.Lc * p.G) * sizeof(float) +
               (size_t)(2 * p.Lc + S) * sizeof(int);
  const size_t vbytes = (size_t)K * D * sizeof(float);
  p.stage_v = aligned16(pooled_value) && (K * D) % 4 == 0 && sm1 + vbytes <= 48 * 1024;
  if (p.stage_v) sm1 += vbytes;
  const size_t sm2 = (size_t)(p.R * p.G + p.Lc * p.G + S * p.G + p.G + p.R) * sizeof(float) +
                     (size_t)(2 * p.Lc + 2 * S) * sizeof(int);
  if (sm1 > 48 * 1024 || sm2 > 48 * 1024)
    return fail(CAST_ERR_UNSUPPORTED, "too large for one CTA (K=%d S=%d rows=%d sketch_groups=%d)", K,
                S, p.R, p.G);
  const SwapLayout lay = swap_layout(p);
  if (!workspace || workspace_bytes < lay.total)
    return fail(CAST_ERR_WORKSPACE, "workspace %zu bytes < required %zu", workspace_bytes, lay.total);
  if (!aligned16(workspace)) return fail(CAST_ERR_ALIGNMENT, "workspace must be 16-byte aligned");
  int st = current_device_sm100(nullptr);
  if (st) return st;
  char *ws = static_cast<char *>(workspace);
  int *cand = reinterpret_cast<int *>(ws + lay.cand);
  float *proxy = reinterpret_cast<float *>(ws + lay.proxy);
  float *err = reinterpret_cast<float *>(ws + lay.err);
  int *limit = reinterpret_cast<int *>(ws + lay.limit);
  auto *best = reinterpret_cast<castk::SwapBest *>(ws + lay.best);
  double *obj = reinterpret_cast<double *>(ws + lay.obj);
  auto *ctl = reinterpret_cast<castk::SwapCtl *>(ws + lay.ctl);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int rows = B * H * p.R;
  CAST_CUDA_TRY(cudaMemsetAsync(ctl, 0, sizeof(castk::SwapCtl), s));
  castk::swap_proxy_kernel<<<rows, castk::kSwapProxyThreads, sm1, s>>>(
      score, pooled_value, selected, counts, local, p, 1e-6f, cand, proxy, err, limit, ctl, gate);
  CAST_CUDA_TRY(cudaGetLastError());
  // rounds: the first also records the objective before any swap; a last
  // pass records the objective after and writes the stats
  if (num_swap_rounds == 0) {
    castk::swap_round_kernel<<<rows, castk::kSwapRoundThreads, sm2, s>>>(
        selected, counts, local, row_gate, coefficient, hessian, p, cand, proxy, err, limit, best, obj,
        ctl, stats, 0, 0, 0, swap_eps, max_swaps_per_call, gate);
    CAST_CUDA_TRY(cudaGetLastError());
  }
  for (int r = 0; r < num_swap_rounds; ++r) {
    castk::swap_round_kernel<<<rows, castk::kSwapRoundThreads, sm2, s>>>(
        selected, counts, local, row_gate, coefficient, hessian, p, cand, proxy, err, limit, best, obj,
        ctl, stats, 1, r == 0 ? 0 : -1, 0, swap_eps, max_swaps_per_call, gate);
    CAST_CUDA_TRY(cudaGetLastError());
  }
  castk::swap_round_kernel<<<rows, castk::kSwapRoundThreads, sm2, s>>>(
      selected, counts, local, row_gate, coefficient, hessian, p, cand, proxy, err, limit, best, obj,
      ctl, stats, 0, 1, 1, swap_eps, max_swaps_per_call, gate);
  CAST_CUDA_TRY(cudaGetLastError());
  return CAST_OK;
}

// ===========================================================================
// PAR / FC-PASM
// ===========================================================================
static int par_chunks(int C) { return ceil_div(C, castk::kParChunk); }

// Per device: the class rfft2 images in castk::g_par_dft (built once), and a
// side stream with two events on which the active-frame copies run beside
// the PAR kernels.  g_par_mutex serialises each call's launch sequence, so
// concurrent callers never interleave on the shared stream and events (nor
// pull the side stream into another caller's stream capture).
static constexpr int kParMaxDevices = 64;
static std::mutex g_par_mutex;
static bool g_par_dft_built[kParMaxDevices] = {};
static void *g_par_dft_ptr[kParMaxDevices] = {};
static cudaStream_t g_par_side[kParMaxDevices] = {};
static cudaEvent_t g_par_fork[kParMaxDevices] = {}, g_par_join[kParMaxDevices] = {};

// Creates the current device's side stream and events, and looks up the
// image array; with g_par_mutex held.
static int par_device_state(int *dev_out) {
  int dev = 0;
  CAST_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kParMaxDevices) return fail(CAST_ERR_UNSUPPORTED, "device %d", dev);
  if (!g_par_side[dev]) {
    CAST_CUDA_TRY(cudaStreamCreateWithFlags(&g_par_side[dev], cudaStreamNonBlocking));
    CAST_CUDA_TRY(cudaEventCreateWithFlags(&g_par_fork[dev], cudaEventDisableTiming));
    CAST_CUDA_TRY(cudaEventCreateWithFlags(&g_par_join[dev], cudaEventDisableTiming));
  }
  if (!g_par_dft_ptr[dev]) CAST_CUDA_TRY(cudaGetSymbolAddress(&g_par_dft_ptr[dev], castk::g_par_dft));
  *dev_out = dev;
  return CAST_OK;
}

extern "C" size_t cast_par_fcpasm_workspace_bytes(int T, int H, int W, int C) {
  if (T <= 0 || H != castk::kParH || W != castk::kParW || C <= 0) return 0;
  const int nt = std::min(T, castk::kParMaxTargets);
  const size_t partials = (size_t)castk::kParMaxPairs * castk::kParTiles * par_chunks(C) * castk::kParPartial;
  const size_t weights = (size_t)nt * castk::kParTiles * castk::kParFreq * 4;
  const size_t pred = (size_t)nt * castk::kParTiles * castk::kParPix * C;
  const size_t filters = (size_t)nt * castk::kParTiles * castk::kParFilterBytes;
  return align_up(partials * 4, 256) + align_up(weights * 4, 256) + align_up(pred * 4, 256) +
         align_up(filters, 1024);
}

static void fill_par_tables(castk::ParTables &t, float tau_low, float tau_high, float power) {
  const double pi = 3.14159265358979323846;
  double hh[castk::kParTH], hw[castk::kParTW];
  for (int i = 0; i < castk::kParTH; ++i) hh[i] = 0.5 - 0.5 * std::cos(2.0 * pi * i / (castk::kParTH - 1));
  for (int j = 0; j < castk::kParTW; ++j) hw[j] = 0.5 - 0.5 * std::cos(2.0 * pi * j / (castk::kParTW - 1));
  for (int i = 0; i < castk::kParTH; ++i)
    for (int j = 0; j < castk::kParTW; ++j) {
      // torch computes the window in float32: outer product then sqrt.
      const float prod = (float)hh[i] * (float)hw[j];
      t.win[i * castk::kParTW + j] = std::sqrt(std::max(prod, 0.0f));
    }
  for (int k = 0; k < castk::kParTW; ++k) {
    t.cw[k] = (float)std::cos(2.0 * pi * k / castk::kParTW);
    t.sw[k] = (float)std::sin(2.0 * pi * k / castk::kParTW);
  }
  for (int k = 0; k < castk::kParTH; ++k) {
    t.ch[k] = (float)std::cos(2.0 * pi * k / castk::kParTH);
    t.shh[k] = (float)std::sin(2.0 * pi * k / castk::kParTH);
  }
  double fy[castk::kParTH], fx[castk::kParWF], rmax = 0.0;
  for (int k = 0; k < castk::kParTH; ++k) {
    const int kk = k <= (castk::kParTH - 1) / 2 ? k : k - castk::kParTH;
    fy[k] = (double)kk / castk::kParTH;
    t.fy[k] = (float)(2.0 * pi * fy[k]);
  }
  for (int k = 0; k < castk::kParWF; ++k) {
    fx[k] = (double)k / castk::kParTW;
    t.fx[k] = (float)(2.0 * pi * fx[k]);
  }
  double r[castk::kParFreq];
  for (int a = 0; a < castk::kParTH; ++a)
    for (int b = 0; b < castk::kParWF; ++b) {
      r[a * castk::kParWF + b] = std::sqrt(fy[a] * fy[a] + fx[b] * fx[b]);
      rmax = std::max(rmax, r[a * castk::kParWF + b]);
    }
  for (int f = 0; f < castk::kParFreq; ++f)
    t.thr[f] = (float)(tau_low + (tau_high - tau_low) * std::pow(r[f] / std::max(rmax, 1e-8), power));
}

extern "C" int cast_par_fcpasm(void *full_residual, const void *active_residual,
                               const int32_t *active_frames, int n_active, int T,
                               int memory_length, int H, int W, int C, float tau_low,
                               float tau_high, float freq_power, float temperature,
                               int ramp_confidence, int current_anchor_boundary,
                               const float *tile_confidence, float *stats_out, void *workspace,
                               size_t workspace_bytes, cast_stream_t stream) {
  if (!full_residual || !active_residual || !active_frames)
    return fail(CAST_ERR_INVALID_ARGUMENT, "full_residual, active_residual, active_frames required");
  if (H != castk::kParH || W != castk::kParW)
    return fail(CAST_ERR_UNSUPPORTED, "PAR grid %dx%d (supported: 22x40, 3x6 tiles of 11x10)", H, W);
  if (C <= 0 || C % 4 || n_active <= 0 || T <= 0 || memory_length < 0 || memory_length > T)
    return fail(CAST_ERR_INVALID_ARGUMENT, "bad sizes (C=%d, n_active=%d, T=%d, memory=%d)", C,
                n_active, T, memory_length);
  if (!(temperature > 0.0f) || !(0.0f <= tau_low && tau_low <= tau_high && tau_high <= 1.0f) ||
      !(freq_power > 0.0f))
    return fail(CAST_ERR_INVALID_ARGUMENT, "invalid FC knobs");
  if (!aligned16(full_residual) || !aligned16(active_residual))
    return fail(CAST_ERR_ALIGNMENT, "residual tensors must be 16-byte aligned");
  for (int i = 0; i < n_active; ++i) {
    if (active_frames[i] < 0 || active_frames[i] >= T)
      return fail(CAST_ERR_INVALID_ARGUMENT, "active frame %d out of range", active_frames[i]);
    if (i && active_frames[i] <= active_frames[i - 1])
      return fail(CAST_ERR_INVALID_ARGUMENT, "active frames must be sorted and unique");
  }
  // Anchors: current-chunk active frames (local ids), as
  // _correct_frequency_confidence_pasm_reference builds exact_local.
  std::vector<int> anchor_row, anchor_local;
  for (int i = 0; i < n_active; ++i)
    if (active_frames[i] >= memory_length) {
      anchor_row.push_back(i);
      anchor_local.push_back(active_frames[i] - memory_length);
    }
  if (anchor_local.empty()) return fail(CAST_ERR_INVALID_ARGUMENT, "FC-PASM requires current anchors");
  const int cur_len = T - memory_length;
  castk::ParParams p;
  memset(&p, 0, sizeof(p));
  // Segment-local bracket rule; pairs in chronological order of first use.
  std::vector<std::pair<int, int>> pairs;
  int nt = 0;
  for (int t = 0; t < cur_len; ++t) {
    bool is_anchor = false;
    for (int a : anchor_local) is_anchor |= (a == t);
    if (is_anchor) continue;
    const bool same = t < current_anchor_boundary;
    int li = -1, ri = -1;
    for (size_t i = 0; i < anchor_local.size(); ++i) {
      const int f = anchor_local[i];
      if ((f < current_anchor_boundary) != same) continue;
      if (f < t) li = (int)i;
      if (f > t && ri < 0) ri = (int)i;
    }
    if (li < 0 || ri < 0) continue;
    int pi = -1;
    for (size_t k2 = 0; k2 < pairs.size(); ++k2)
      if (pairs[k2].first == li && pairs[k2].second == ri) pi = (int)k2;
    if (pi < 0) {
      if ((int)pairs.size() == castk::kParMaxPairs) return fail(CAST_ERR_UNSUPPORTED, "too many anchor pairs");
      pairs.push_back({li, ri});
      pi = (int)pairs.size() - 1;
    }
    if (nt == castk::kParMaxTargets) return fail(CAST_ERR_UNSUPPORTED, "too many targets");
    p.target_pair[nt] = pi;
    p.target_frame[nt] = memory_length + t;
    p.target_alpha[nt] = (float)((double)(t - anchor_local[li]) / (double)(anchor_local[ri] - anchor_local[li]));
    ++nt;
  }
  const size_t need = cast_par_fcpasm_workspace_bytes(T, H, W, C);
  if (!workspace || workspace_bytes < need)
    return fail(CAST_ERR_WORKSPACE, "workspace %zu bytes < required %zu", workspace_bytes, need);
  int num_sms = 0;
  int st = current_device_sm100(&num_sms);
  if (st) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const size_t frame_bytes = (size_t)H * W * C * 2;
  __nv_bfloat16 *full = static_cast<__nv_bfloat16 *>(full_residual);
  const __nv_bfloat16 *act = static_cast<const __nv_bfloat16 *>(active_residual);

  std::lock_guard<std::mutex> lock(g_par_mutex);
  int dev = 0;
  if ((st = par_device_state(&dev))) return st;
  // corrected[:, active_frames] = active_residual: independent of the target
  // frames, so with targets present the copies run on the side stream beside
  // the PAR kernels and `s` waits for them at the end
  const bool fork = nt > 0;
  cudaStream_t cs = s;
  if (fork) {
    CAST_CUDA_TRY(cudaEventRecord(g_par_fork[dev], s));
    CAST_CUDA_TRY(cudaStreamWaitEvent(g_par_side[dev], g_par_fork[dev], 0));
    cs = g_par_side[dev];
  }
  for (int i = 0; i < n_active; ++i) {
    void *dst = full + (size_t)active_frames[i] * H * W * C;
    const void *src = act + (size_t)i * H * W * C;
    if (dst != src) CAST_CUDA_TRY(cudaMemcpyAsync(dst, src, frame_bytes, cudaMemcpyDeviceToDevice, cs));
  }
  if (fork) CAST_CUDA_TRY(cudaEventRecord(g_par_join[dev], cs));

  if (nt > 0) {
    p.active = act;
    p.full = full;
    p.C = C;
    p.HW = H * W;
    p.n_chunks = par_chunks(C);
    p.n_pairs = (int)pairs.size();
    p.n_targets = nt;
    for (size_t i = 0; i < pairs.size(); ++i) {
      p.pair_left[i] = anchor_row[pairs[i].first];
      p.pair_right[i] = anchor_row[pairs[i].second];
    }
    p.temperature = temperature;
    p.ramp_confidence = ramp_confidence;
    p.tile_confidence = tile_confidence;
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    p.partials = reinterpret_cast<float *>(ws);
    ws += align_up((size_t)castk::kParMaxPairs * castk::kParTiles * p.n_chunks * castk::kParPartial * 4, 256);
    p.weights = reinterpret_cast<float *>(ws);
    ws += align_up((size_t)std::min(T, castk::kParMaxTargets) * castk::kParTiles * castk::kParFreq * 16, 256);
    p.pred = reinterpret_cast<float *>(ws);
    ws += align_up((size_t)std::min(T, castk::kParMaxTargets) * castk::kParTiles * castk::kParPix * C * 4, 256);
    p.filters = ws;
    p.dft = static_cast<uint8_t *>(g_par_dft_ptr[dev]);
    p.stats = stats_out;
    fill_par_tables(p.tab, tau_low, tau_high, freq_power);

    static std::once_flag once;
    static cudaError_t aerr = cudaSuccess;
    const int smem_stats = 4 * castk::kParFreq * (castk::kParChunk + 1) * 4;
    const int smem_pred = 6 * castk::kParFreq * (castk::kParChunk + 1) * 4;
    std::call_once(once, [&] {
      aerr = cudaFuncSetAttribute(castk::par_stats_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_stats);
      if (aerr == cudaSuccess)
        aerr = cudaFuncSetAttribute(castk::par_predict_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_pred);
    });
    CAST_CUDA_TRY(aerr);
    // Tensor-core paths when every 8-channel group is a 16-byte aligned copy
    // (statistics and prediction) and a pair's targets fit the TMEM columns
    // (prediction); the per-channel DFT kernels otherwise.
    const bool mma_ok = C % 8 == 0 && reinterpret_cast<uintptr_t>(act) % 16 == 0;
    int max_per_pair = 0;
    for (int i = 0; i < p.n_pairs; ++i) {
      int cnt = 0;
      for (int t = 0; t < nt; ++t) cnt += p.target_pair[t] == i;
      max_per_pair = std::max(max_per_pair, cnt);
    }
    if (mma_ok) {
      static std::once_flag mma_once;
      static cudaError_t mma_err = cudaSuccess;
      std::call_once(mma_once, [] {
        mma_err = cudaFuncSetAttribute(castk::par_predict_mma_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       castk::ParMmaSmem::alloc);
        if (mma_err == cudaSuccess)
          mma_err = cudaFuncSetAttribute(castk::par_stats_mma_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         castk::ParStatSmem::alloc);
      });
      CAST_CUDA_TRY(mma_err);
    }
    dim3 g1(p.n_chunks, castk::kParTiles, p.n_pairs);
    // anchor frames as (channel, column, row, frame); one box of 64 channels
    // x 10 columns x 11 rows per tile, anchor and channel half
    CUtensorMap tm_act;
    if (mma_ok && (st = make_map_4d(&tm_act, act, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, C, W, H, n_active, 64,
                                    castk::kParTW, castk::kParTH, CU_TENSOR_MAP_SWIZZLE_128B)))
      return st;
    if (mma_ok) {
      p.n_stat_chunks = ceil_div(C, 128);
      // CTAs per tile class in proportion to its items, at least one each
      int n_cls[castk::kParClasses], g_cls[castk::kParClasses];
      long long total = 0;
      for (int c = 0; c < castk::kParClasses; ++c) {
        n_cls[c] = castk::par_class_tiles(c) * p.n_pairs * p.n_stat_chunks;
        total += n_cls[c];
      }
      const int grid = (int)std::max<long long>(castk::kParClasses, std::min<long long>(num_sms, total));
      int sum = 0;
      for (int c = 0; c < castk::kParClasses; ++c) {
        g_cls[c] = (int)std::max<long long>(1, (long long)grid * n_cls[c] / total);
        sum += g_cls[c];
      }
      while (sum > grid) {  // take from the class with the most CTAs
        int big = 0;
        for (int c = 1; c < castk::kParClasses; ++c) big = g_cls[c] > g_cls[big] ? c : big;
        --g_cls[big];
        --sum;
      }
      while (sum < grid) {  // give to the class with the most items per CTA
        int need = 0;
        for (int c = 1; c < castk::kParClasses; ++c)
          need = (long long)n_cls[c] * g_cls[need] > (long long)n_cls[need] * g_cls[c] ? c : need;
        ++g_cls[need];
        ++sum;
      }
      p.stat_cta_start[0] = 0;
      for (int c = 0; c < castk::kParClasses; ++c) p.stat_cta_start[c + 1] = p.stat_cta_start[c] + g_cls[c];
      const dim3 dft_grid(ceil_div(castk::kParN * (castk::kParN / 8), 256), castk::kParClasses);
      if (!g_par_dft_built[dev]) {
        cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
        CAST_CUDA_TRY(cudaStreamIsCapturing(s, &capture));
        if (capture == cudaStreamCaptureStatusNone) {
          // once per device, on the private stream (no wait on the caller's)
          castk::par_dft_kernel<<<dft_grid, 256, 0, g_par_side[dev]>>>(p);
          CAST_CUDA_TRY(cudaGetLastError());
          CAST_CUDA_TRY(cudaStreamSynchronize(g_par_side[dev]));
          g_par_dft_built[dev] = true;
        } else {
          // inside a capture nothing may synchronise: the graph builds them
          castk::par_dft_kernel<<<dft_grid, 256, 0, s>>>(p);
          CAST_CUDA_TRY(cudaGetLastError());
        }
      }
      castk::par_stats_mma_kernel<<<grid, castk::kParStatThreads, castk::ParStatSmem::alloc, s>>>(tm_act, p);
    } else {
      p.n_stat_chunks = p.n_chunks;
      castk::par_stats_kernel<<<g1, castk::kParChunk, smem_stats, s>>>(p);
    }
    CAST_CUDA_TRY(cudaGetLastError());
    const bool predict_mma = mma_ok && max_per_pair <= castk::kParMmaTargets;
    castk::par_finalize_kernel<<<dim3(castk::kParTiles, p.n_pairs), castk::kParFinalizeThreads, 0, s>>>(p);
    CAST_CUDA_TRY(cudaGetLastError());
    if (predict_mma) {
      castk::par_filter_kernel<<<dim3(castk::kParTiles, nt, castk::kParKChunks), 256, 0, s>>>(p);
      CAST_CUDA_TRY(cudaGetLastError());
      const int n_units = nt * castk::kParTiles * ceil_div(C, 128);
      castk::par_predict_mma_kernel<<<std::min(n_units, num_sms), castk::kParPredThreads,
                                      castk::ParMmaSmem::alloc, s>>>(tm_act, p);
      CAST_CUDA_TRY(cudaGetLastError());
    } else {
      castk::par_predict_kernel<<<g1, castk::kParChunk, smem_pred, s>>>(p);
      CAST_CUDA_TRY(cudaGetLastError());
    }
    castk::par_ola_kernel<<<dim3(H * W, nt), 256, 0, s>>>(p);
    CAST_CUDA_TRY(cudaGetLastError());
  }
  if (fork) CAST_CUDA_TRY(cudaStreamWaitEvent(s, g_par_join[dev], 0));
  return CAST_OK;
}

// ===========================================================================
// allocation-free RCSA selection + quantisation
// ===========================================================================
// One static scratch array per device (each device's copy of this module has
// its own); every call on that device shares it, so calls must not overlap on
// the GPU.  Nothing in it needs to start at zero.
static __device__ __align__(256) uint8_t g_noalloc_scratch[CAST_NOALLOC_SCRATCH_BYTES];

static constexpr int kNoAllocMaxDevices = 64;
static std::mutex g_noalloc_mutex;
static void *g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Address of the current device's scratch, looked up once per device with
// that device current.
static int noalloc_scratch(void **out) {
  int dev = 0;
  CAST_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return fail(CAST_ERR_UNSUPPORTED, "device ordinal %d >= %d", dev, kNoAllocMaxDevices);
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_ptr[dev]) {
    void *ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || !ptr)
      return fail(CAST_ERR_CUDA, "cudaGetSymbolAddress(scratch) on device %d: %s", dev,
                  cudaGetErrorString(e));
    g_noalloc_ptr[dev] = ptr;
  }
  *out = g_noalloc_ptr[dev];
  return CAST_OK;
}

extern "C" int cast_rcsa_select_quant_noalloc(const void *q, const void *k, const void *v,
                                              const uint8_t *q_valid, const uint8_t *k_valid, int B,
                                              int H, int Lq, int Lk, int D, int block_size,
                                              int budget, int rule, int32_t *sel_idx,
                                              int32_t *sel_cnt, int8_t *q_codes, float *q_scales,
                                              int8_t *k_codes, float *k_scales, int8_t *v_codes,
                                              float *v_scales, uint8_t *qk_mode, int policy,
                                              float int8_tolerance, double *pooled,
                                              cast_stream_t stream) {
  const size_t need = cast_rcsa_select_quant_workspace_bytes(B, H, Lq, Lk, D, block_size);
  if (need > CAST_NOALLOC_SCRATCH_BYTES)
    return fail(CAST_ERR_WORKSPACE,
                "needs %zu bytes of scratch; the static scratch holds %zu "
                "(use cast_rcsa_select_quant with a caller workspace)",
                need, (size_t)CAST_NOALLOC_SCRATCH_BYTES);
  int st = current_device_sm100(nullptr);
  if (st) return st;
  void *scratch = nullptr;
  st = noalloc_scratch(&scratch);
  if (st) return st;
  return cast_rcsa_select_quant(q, k, v, q_valid, k_valid, B, H, Lq, Lk, D, block_size, budget, rule, sel_idx,
                                sel_cnt, q_codes, q_scales, k_codes, k_scales, v_codes, v_scales,
                                qk_mode, policy, int8_tolerance, pooled, scratch,
                                CAST_NOALLOC_SCRATCH_BYTES, stream);
}
