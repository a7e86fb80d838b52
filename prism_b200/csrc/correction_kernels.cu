// Bias rectification of the uniform block-sparse path (inference):
// hymm/models/modules/block_sparse_attention/bias_rectification.py:261-446 and its
// fused kernels bias_rectification_triton.py:9-363.
//
// Per (head, q chunk a) the chunk scores give A = softmax over the valid key chunks
// of score * sm_scale (_masked_softmax_along_last, :146-152), the kept mass
// R = max(1 - sum of A over the valid unselected chunks, 1e-6) and the variance M
// of A over the valid chunks (_masked_var_along_last, :155-170).
//   Rectified:  O' = R O_spa + (A * unselected) V_cmp        (:335-377, :421-446)
//   Taylor:     for q chunks with M < quantile(M, alpha_f), O_spa is merged with
//               an attention over the unselected pooled keys K_cmp / V_cmp with
//               score offsets log(valid tokens of the chunk) (:190-257, :300-324);
//               that attention is the forward kernel's key-bias form
//               (prism_bsa_fwd_keybias), the merge is by log-sum-exp.
// Statistics are sums in a fixed order (per-thread strided partials over 256
// threads, then a halving tree) with deterministic exponentials, so the CPU
// oracle reproduces them bit for bit.  Build with -fmad=false.
#include <cuda_bf16.h>
#include <math.h>
#include <stdint.h>

#include "prism_bsa.h"
#include "prism_common.cuh"

namespace prism {

constexpr int kCorrThreads = 256;

// sum over the block of one partial per thread: red[t] += red[t + s] for
// s = 128, 64, ..., 1 (the order the oracle restates)
__device__ float tree_sum256(float v, float* red) {
  red[threadIdx.x] = v;
  __syncthreads();
  for (int s = kCorrThreads / 2; s > 0; s >>= 1) {
    if (threadIdx.x < s) red[threadIdx.x] = __fadd_rn(red[threadIdx.x], red[threadIdx.x + s]);
    __syncthreads();
  }
  const float r = red[0];
  __syncthreads();
  return r;
}

__device__ __forceinline__ bool chunk_has_key(const uint64_t* tile_bits, int j, int tk) {
  for (int i = 0; i < tk; ++i)
    if (tile_bits[(int64_t)j * tk + i] != 0ull) return true;
  return false;
}

__device__ __forceinline__ bool chunk_selected(const uint32_t* row, int j, int tk) {
  for (int i = 0; i < tk; ++i) {
    const int t = j * tk + i;
    if ((row[t >> 5] >> (t & 31)) & 1u) return true;
  }
  return false;
}

// One CTA per (q chunk a, head h).  scores [h][nq][nk] raw chunk scores; bits_q the
// selection's tile bitmap (q tile a*tq's row; a key chunk is selected iff one of its
// tk tiles is set); tile_bits the key validity (a chunk is valid iff one of its
// tiles holds a valid key).  Dynamic shared memory: nk floats (the exponentials).
__global__ void __launch_bounds__(kCorrThreads) correction_stats_kernel(
    const float* __restrict__ scores, int nq, int nk, int tq, int tk, const uint32_t* __restrict__ bits_q,
    int64_t n_qt, int wk, const uint64_t* __restrict__ tile_bits, float sm_scale, float* __restrict__ R,
    float* __restrict__ M, uint64_t* __restrict__ nonsel, float* __restrict__ a_rect) {
  extern __shared__ float e[];
  __shared__ float red[kCorrThreads];
  __shared__ int cnt_sh;
  const int a = blockIdx.x, h = blockIdx.y, t = threadIdx.x;
  const float* s = scores + ((int64_t)h * nq + a) * nk;
  const uint32_t* row = bits_q + ((int64_t)h * n_qt + (int64_t)a * tq) * wk;
  const int wn = (nk + 63) / 64;
  // pass 1: x = score * scale on valid chunks, maximum
  float mx = -INFINITY;
  int cnt = 0;
  for (int j = t; j < nk; j += kCorrThreads) {
    const bool v = chunk_has_key(tile_bits, j, tk);
    const float x = v ? __fmul_rn(s[j], sm_scale) : -INFINITY;
    e[j] = x;
    mx = fmaxf(mx, x);
    cnt += v;
  }
  if (t == 0) cnt_sh = 0;
  for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((t & 31) == 0) red[t >> 5] = mx;
  __syncthreads();
  atomicAdd(&cnt_sh, cnt);
  if (t < 32) {
    float m2 = t < kCorrThreads / 32 ? red[t] : -INFINITY;
    for (int o = 16; o >= 1; o >>= 1) m2 = fmaxf(m2, __shfl_xor_sync(0xffffffffu, m2, o));
    if (t == 0) red[0] = m2;
  }
  __syncthreads();
  mx = red[0];
  const int n_valid = cnt_sh;
  __syncthreads();
  // pass 2: exponentials and their sum
  float part = 0.0f;
  for (int j = t; j < nk; j += kCorrThreads) {
    const float x = e[j];
    const float ex = x == -INFINITY ? 0.0f : det_expf(__fsub_rn(x, mx));
    e[j] = ex;
    part = __fadd_rn(part, ex);
  }
  const float sum = tree_sum256(part, red);
  // pass 3: A, the unselected valid mass, the mean of A over valid chunks
  float prect = 0.0f, pmean = 0.0f;
  for (int j = t; j < nk; j += kCorrThreads) {
    const float A = __fdiv_rn(e[j], sum);
    e[j] = A;
    const bool v = chunk_has_key(tile_bits, j, tk);
    const bool rect = v && !chunk_selected(row, j, tk);
    if (rect) prect = __fadd_rn(prect, A);
    if (v) pmean = __fadd_rn(pmean, A);
    if (a_rect != nullptr) a_rect[((int64_t)h * nq + a) * nk + j] = rect ? A : 0.0f;
  }
  const float rsum = tree_sum256(prect, red);
  const float fn = n_valid > 0 ? (float)n_valid : 1.0f;
  const float mean = __fdiv_rn(tree_sum256(pmean, red), fn);
  float pvar = 0.0f;
  for (int j = t; j < nk; j += kCorrThreads) {
    if (!chunk_has_key(tile_bits, j, tk)) continue;
    const float d = __fsub_rn(e[j], mean);
    pvar = __fadd_rn(pvar, __fmul_rn(d, d));
  }
  const float var = __fdiv_rn(tree_sum256(pvar, red), fn);
  if (t == 0) {
    const float r = __fsub_rn(1.0f, rsum);
    R[(int64_t)h * nq + a] = r < 1e-6f ? 1e-6f : r;
    M[(int64_t)h * nq + a] = var;
  }
  if (nonsel != nullptr) {
    // unselected valid chunks as 64-bit words (bit j & 63 of word j >> 6)
    for (int w = t; w < wn; w += kCorrThreads) {
      uint64_t bitsw = 0;
      for (int i = 0; i < 64; ++i) {
        const int j = w * 64 + i;
        if (j < nk && chunk_has_key(tile_bits, j, tk) && !chunk_selected(row, j, tk))
          bitsw |= 1ull << i;
      }
      nonsel[((int64_t)h * nq + a) * wn + w] = bitsw;
    }
  }
}

// Taylor pass inputs: for head h, q tile t (chunk a = t / tq, rows of real chunks
// only) and pooled-key tile u: masks[h][t][u] = flat(h, a) ? nonsel[h][a][u] : 0,
// flat = M < *tau; bits_t[h][t] bit u = masks[h][t][u] != 0.  One warp per
// (h, t, 32 pooled tiles).
__global__ void taylor_prep_kernel(const uint64_t* __restrict__ nonsel, const float* __restrict__ M,
                                   const float* __restrict__ tau, int heads, int64_t n_qt, int tq,
                                   int nq, int n_ut, int wn, int wt, uint64_t* __restrict__ masks,
                                   uint32_t* __restrict__ bits_t) {
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t per_head = n_qt * wt;
  if (gw >= (int64_t)heads * per_head) return;
  const int h = (int)(gw / per_head);
  const int64_t t = (gw % per_head) / wt;
  const int wi = (int)(gw % wt);
  const int u = wi * 32 + lane;
  const int a = (int)(t / tq);
  uint64_t m = 0;
  if (a < nq && u < n_ut && u < wn && M[(int64_t)h * nq + a] < *tau)
    m = nonsel[((int64_t)h * nq + a) * wn + u];
  if (u < n_ut) masks[((int64_t)h * n_qt + t) * n_ut + u] = m;
  const uint32_t b = __ballot_sync(0xffffffffu, m != 0ull);
  if (lane == 0) bits_t[((int64_t)h * n_qt + t) * wt + wi] = b;
}

// Score offsets of the pooled keys: log(valid tokens of chunk j, at least 1) /
// sm_scale for j < nk, 0 for the padding rows up to n_pad.
__global__ void key_log_bias_kernel(const uint64_t* __restrict__ tile_bits, int nk, int tk, int n_pad,
                                    float sm_scale, float* __restrict__ bias) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n_pad) return;
  float b = 0.0f;
  if (j < nk) {
    int c = 0;
    for (int i = 0; i < tk; ++i) c += __popcll(tile_bits[(int64_t)j * tk + i]);
    b = logf(c > 1 ? (float)c : 1.0f) / sm_scale;
  }
  bias[j] = b;
}

// fp32 rows [heads][n][D] -> bf16 rows [heads][n_pad][D], zero rows past n.
__global__ void rows_to_bf16_kernel(const float* __restrict__ x, int heads, int n, int D, int n_pad,
                                    __nv_bfloat16* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)heads * n_pad * D;
  if (i >= total) return;
  const int d = (int)(i % D);
  const int64_t r = (i / D) % n_pad;
  const int h = (int)(i / ((int64_t)D * n_pad));
  out[i] = __float2bfloat16_rn(r < n ? x[((int64_t)h * n + r) * D + d] : 0.0f);
}

__device__ __forceinline__ float o_f32(const __nv_bfloat16* hi, const __nv_bfloat16* lo, int64_t i) {
  const float v = __bfloat162float(hi[i]);
  return lo != nullptr ? v + __bfloat162float(lo[i]) : v;
}

// out = flat(h, a) ? w_spa O_spa + w_t O_t : O_spa (_taylor_merge_fwd_kernel's merge,
// bias_rectification_triton.py:270-292); rows in chunk order, a = row / chunk_q.
// One warp per row.
__global__ void taylor_merge_kernel(const __nv_bfloat16* __restrict__ o_spa,
                                    const __nv_bfloat16* __restrict__ o_spa_lo,
                                    const float* __restrict__ lse_spa, const __nv_bfloat16* __restrict__ o_t,
                                    const __nv_bfloat16* __restrict__ o_t_lo,
                                    const float* __restrict__ lse_t, const float* __restrict__ M,
                                    const float* __restrict__ tau, int heads, int64_t S, int64_t seq_q,
                                    int chunk_q, int nq, int D, __nv_bfloat16* __restrict__ out) {
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= (int64_t)heads * S) return;
  const int h = (int)(gw / S);
  const int64_t r = gw % S;
  const int64_t base = gw * D;
  bool flat = false;
  if (r < seq_q) flat = M[(int64_t)h * nq + r / chunk_q] < *tau;
  float ws = 1.0f, wt = 0.0f;
  if (flat) {
    const float ls = lse_spa[gw], lt = lse_t[gw];
    const float lm = fmaxf(ls, lt);
    if (lm > -INFINITY) {  // lse_total = max + log(e^(a - max) + e^(b - max)); exp(-inf) = 0
      const float tot = lm + logf(expf(ls - lm) + expf(lt - lm));
      ws = expf(ls - tot);
      wt = expf(lt - tot);
    }
  }
  for (int d = lane; d < D; d += 32) {
    float v = o_f32(o_spa, o_spa_lo, base + d);
    if (flat) v = ws * v + wt * o_f32(o_t, o_t_lo, base + d);
    out[base + d] = __float2bfloat16_rn(v);
  }
}

// o_ncri[h][a][d] = sum over key chunks j (in order) of a_rect[h][a][j] * v_cmp[h][j][d]:
// the unselected chunks' pooled-softmax mass times their pooled values (the A_rect
// V_cmp of _rectified_correction_fwd_kernel, bias_rectification_triton.py:9-95).
// CTA = 64 q chunks x 64 channels of one head, 256 threads with 4 x 4 outputs each;
// the reduction runs over kRectK key chunks at a time staged in shared memory, one
// fmaf per (output, j) in increasing j, so the result is deterministic.
constexpr int kRectTile = 64, kRectK = 32;
__global__ void __launch_bounds__(256) rect_contract_kernel(const float* __restrict__ a_rect,
                                                            const float* __restrict__ v_cmp, int nq,
                                                            int nk, int D, float* __restrict__ out) {
  __shared__ float As[kRectK][kRectTile + 4];  // [j][a]
  __shared__ float Vs[kRectK][kRectTile + 4];  // [j][d]
  const int a0 = blockIdx.y * kRectTile, d0 = blockIdx.x * kRectTile, h = blockIdx.z;
  const float* ah = a_rect + (int64_t)h * nq * nk;
  const float* vh = v_cmp + (int64_t)h * nk * D;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
  for (int j0 = 0; j0 < nk; j0 += kRectK) {
    for (int i = threadIdx.x; i < kRectK * kRectTile; i += blockDim.x) {
      const int r = i / kRectK, j = i % kRectK;  // A: row r (q chunk), column j (coalesced in j)
      As[j][r] = (a0 + r < nq && j0 + j < nk) ? ah[(int64_t)(a0 + r) * nk + j0 + j] : 0.0f;
      const int jj = i / kRectTile, c = i % kRectTile;  // V: row jj (key chunk), channel c
      Vs[jj][c] = (j0 + jj < nk && d0 + c < D) ? vh[(int64_t)(j0 + jj) * D + d0 + c] : 0.0f;
    }
    __syncthreads();
    const int jn = min(kRectK, nk - j0);
    for (int j = 0; j < jn; ++j) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[j][ty * 4 + i];
#pragma unroll
      for (int k = 0; k < 4; ++k) bv[k] = Vs[j][tx * 4 + k];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int k = 0; k < 4; ++k) acc[i][k] = __fmaf_rn(av[i], bv[k], acc[i][k]);
    }
    __syncthreads();
  }
  float* oh = out + (int64_t)h * nq * D;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int a = a0 + ty * 4 + i;
    if (a >= nq) continue;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int d = d0 + tx * 4 + k;
      if (d < D) oh[(int64_t)a * D + d] = acc[i][k];
    }
  }
}

// out = R(h, a) O_spa + O_ncri(h, a) (_rectified_correction_fwd_kernel,
// bias_rectification_triton.py:9-95); rows in chunk order past seq_q copy O_spa.
__global__ void rectified_apply_kernel(const __nv_bfloat16* __restrict__ o_spa,
                                       const __nv_bfloat16* __restrict__ o_spa_lo,
                                       const float* __restrict__ R, const float* __restrict__ o_ncri,
                                       int heads, int64_t S, int64_t seq_q, int chunk_q, int nq, int D,
                                       __nv_bfloat16* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)heads * S * D) return;
  const int d = (int)(i % D);
  const int64_t r = (i / D) % S;
  const int h = (int)(i / ((int64_t)D * S));
  float v = o_f32(o_spa, o_spa_lo, i);
  if (r < seq_q) {
    const int64_t a = (int64_t)h * nq + r / chunk_q;
    v = R[a] * v + o_ncri[a * D + d];
  }
  out[i] = __float2bfloat16_rn(v);
}

}  // namespace prism

using namespace prism;

extern "C" {

prism_status_t prism_correction_stats(const float* scores, int heads, int nq, int nk, int tq, int tk,
                                      const uint32_t* bits_q, int64_t n_qt, int64_t n_kt,
                                      const uint64_t* tile_bits, float sm_scale, float* R, float* M,
                                      uint64_t* nonsel, float* a_rect, cudaStream_t stream) {
  PRISM_CHECK_ARG(scores && bits_q && tile_bits && R && M, "prism_correction_stats: null pointer");
  PRISM_CHECK_ARG(heads >= 1 && nq >= 1 && nk >= 1 && tq >= 1 && tk >= 1,
                  "prism_correction_stats: bad sizes");
  PRISM_CHECK_ARG((int64_t)nq * tq <= n_qt && (int64_t)nk * tk <= n_kt,
                  "prism_correction_stats: chunks exceed the tile bitmaps");
  const size_t smem = (size_t)nk * sizeof(float);
  PRISM_CHECK_ARG(smem <= 200 * 1024, "prism_correction_stats: %d key chunks exceed shared memory", nk);
  PRISM_CHECK_CUDA(cudaFuncSetAttribute(correction_stats_kernel,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                   "prism_correction_stats: smem attribute");
  const int wk = (int)((n_kt + 31) / 32);
  correction_stats_kernel<<<dim3(nq, heads), kCorrThreads, smem, stream>>>(
      scores, nq, nk, tq, tk, bits_q, n_qt, wk, tile_bits, sm_scale, R, M, nonsel, a_rect);
  PRISM_CHECK_LAUNCH("prism_correction_stats");
  return PRISM_OK;
}

prism_status_t prism_taylor_prep(const uint64_t* nonsel, const float* M, const float* tau, int heads,
                                 int64_t n_qt, int tq, int nq, int nk, int64_t n_ut, uint64_t* masks,
                                 uint32_t* bits_t, cudaStream_t stream) {
  PRISM_CHECK_ARG(nonsel && M && tau && masks && bits_t, "prism_taylor_prep: null pointer");
  PRISM_CHECK_ARG(heads >= 1 && tq >= 1 && nq >= 1 && (int64_t)nq * tq <= n_qt && n_ut >= 1 &&
                      nk <= n_ut * 64,
                  "prism_taylor_prep: bad sizes");
  const int wn = (nk + 63) / 64;
  const int wt = (int)((n_ut + 31) / 32);
  const int64_t warps = (int64_t)heads * n_qt * wt;
  taylor_prep_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, stream>>>(
      nonsel, M, tau, heads, n_qt, tq, nq, (int)n_ut, wn, wt, masks, bits_t);
  PRISM_CHECK_LAUNCH("prism_taylor_prep");
  return PRISM_OK;
}

prism_status_t prism_key_log_bias(const uint64_t* tile_bits, int nk, int tk, int n_pad, float sm_scale,
                                  float* bias, cudaStream_t stream) {
  PRISM_CHECK_ARG(tile_bits && bias, "prism_key_log_bias: null pointer");
  PRISM_CHECK_ARG(nk >= 1 && tk >= 1 && n_pad >= nk && sm_scale > 0.0f, "prism_key_log_bias: bad sizes");
  key_log_bias_kernel<<<(n_pad + 255) / 256, 256, 0, stream>>>(tile_bits, nk, tk, n_pad, sm_scale, bias);
  PRISM_CHECK_LAUNCH("prism_key_log_bias");
  return PRISM_OK;
}

prism_status_t prism_rows_to_bf16(const float* x, int heads, int n, int D, int n_pad, void* out,
                                  cudaStream_t stream) {
  PRISM_CHECK_ARG(x && out, "prism_rows_to_bf16: null pointer");
  PRISM_CHECK_ARG(heads >= 1 && n >= 0 && D >= 1 && n_pad >= n, "prism_rows_to_bf16: bad sizes");
  const int64_t total = (int64_t)heads * n_pad * D;
  if (total == 0) return PRISM_OK;
  rows_to_bf16_kernel<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>(x, heads, n, D, n_pad,
                                                                          (__nv_bfloat16*)out);
  PRISM_CHECK_LAUNCH("prism_rows_to_bf16");
  return PRISM_OK;
}

prism_status_t prism_taylor_merge(const void* o_spa, const void* o_spa_lo, const float* lse_spa,
                                  const void* o_t, const void* o_t_lo, const float* lse_t,
                                  const float* M, const float* tau, int heads, int64_t S, int64_t seq_q,
                                  int chunk_q, int D, void* out, cudaStream_t stream) {
  PRISM_CHECK_ARG(o_spa && lse_spa && o_t && lse_t && M && tau && out, "prism_taylor_merge: null pointer");
  PRISM_CHECK_ARG(heads >= 1 && S >= seq_q && seq_q >= 1 && chunk_q >= 1 && seq_q % chunk_q == 0 && D >= 1,
                  "prism_taylor_merge: bad sizes");
  const int64_t warps = (int64_t)heads * S;
  taylor_merge_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, stream>>>(
      (const __nv_bfloat16*)o_spa, (const __nv_bfloat16*)o_spa_lo, lse_spa, (const __nv_bfloat16*)o_t,
      (const __nv_bfloat16*)o_t_lo, lse_t, M, tau, heads, S, seq_q, chunk_q, (int)(seq_q / chunk_q), D,
      (__nv_bfloat16*)out);
  PRISM_CHECK_LAUNCH("prism_taylor_merge");
  return PRISM_OK;
}

prism_status_t prism_rectified_apply(const void* o_spa, const void* o_spa_lo, const float* R,
                                     const float* o_ncri, int heads, int64_t S, int64_t seq_q, int chunk_q,
                                     int D, void* out, cudaStream_t stream) {
  PRISM_CHECK_ARG(o_spa && R && o_ncri && out, "prism_rectified_apply: null pointer");
  PRISM_CHECK_ARG(heads >= 1 && S >= seq_q && seq_q >= 1 && chunk_q >= 1 && seq_q % chunk_q == 0 && D >= 1,
                  "prism_rectified_apply: bad sizes");
  const int64_t total = (int64_t)heads * S * D;
  rectified_apply_kernel<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>(
      (const __nv_bfloat16*)o_spa, (const __nv_bfloat16*)o_spa_lo, R, o_ncri, heads, S, seq_q, chunk_q,
      (int)(seq_q / chunk_q), D, (__nv_bfloat16*)out);
  PRISM_CHECK_LAUNCH("prism_rectified_apply");
  return PRISM_OK;
}

prism_status_t prism_rectified_contract(const float* a_rect, const float* v_cmp, int heads, int nq, int nk,
                                        int D, float* o_ncri, cudaStream_t stream) {
  PRISM_CHECK_ARG(a_rect && v_cmp && o_ncri, "prism_rectified_contract: null pointer");
  PRISM_CHECK_ARG(heads >= 1 && heads <= 65535 && nq >= 1 && nk >= 1 && D >= 1,
                  "prism_rectified_contract: bad sizes");
  rect_contract_kernel<<<dim3((unsigned)((D + kRectTile - 1) / kRectTile),
                              (unsigned)((nq + kRectTile - 1) / kRectTile), heads),
                         256, 0, stream>>>(a_rect, v_cmp, nq, nk, D, o_ncri);
  PRISM_CHECK_LAUNCH("prism_rectified_contract");
  return PRISM_OK;
}

}  // extern "C"
