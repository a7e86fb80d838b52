// Selection side of the dynamic block-sparse attention path: audio token norms,
// zone statistics, per-zone shape choice, permutation / tile maps, row gather
// and scatter, pooled block scoring and hybrid top-k + cumulative-mass
// selection into q-major / k-major tile bitmaps.
//
// Compiled with -fmad=false: every floating-point step is one IEEE operation in
// a fixed order, so results are bit-identical to the CPU restatement in
// oracle/prism_oracle.c and to themselves run after run (the reference
// recomputes the selection under activation checkpointing,
// dynamic_block_attention.py:256-319, so it must be deterministic).
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdarg.h>
#include <stdint.h>

#include "prism_common.cuh"

namespace prism {

static thread_local char g_err[512] = "";
void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}
const char* last_error() { return g_err; }

// ===================================================================== a2
// One warp per token.  Lane l owns 8-element chunks l, l+32, ...; within a
// chunk acc = fma(x, x, acc) in element order; then an xor butterfly.
__global__ void token_norms_kernel(const uint16_t* __restrict__ x, int64_t n, int dim,
                                   __nv_bfloat16* __restrict__ out) {
  const int64_t tok = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (tok >= n) return;
  const uint4* row = reinterpret_cast<const uint4*>(x + tok * (int64_t)dim);
  const int nchunks = dim >> 3;
  float acc = 0.0f;
  for (int c = lane; c < nchunks; c += 32) {
    uint4 u = __ldg(row + c);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float lo = __uint_as_float(w[j] << 16);
      float hi = __uint_as_float(w[j] & 0xffff0000u);
      acc = __fmaf_rn(lo, lo, acc);
      acc = __fmaf_rn(hi, hi, acc);
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
  if (lane == 0) out[tok] = __float2bfloat16_rn(__fsqrt_rn(acc));
}

// ============================================================ a4/a5/a6
// Stage 1: one CTA per (zone, local frame lt); thread i owns channels 2i, 2i+1.
// Partial layout per (zone, lt): [17][D] = frame | rowH[8] | colW[8]; audio
// partial [17] the same for the scalar norm.
constexpr int kPart = 17;

__device__ __forceinline__ bool token_valid(int t, int h, int w, int T, int H, int W, int Hp,
                                            int Wp, const uint8_t* __restrict__ valid,
                                            int64_t& src) {
  if (t >= T || h >= H || w >= W) return false;
  if (valid != nullptr && !valid[((int64_t)t * Hp + h) * Wp + w]) return false;
  src = ((int64_t)t * H + h) * W + w;
  return true;
}

__global__ void zone_partial_kernel(const uint16_t* __restrict__ v, int heads, int64_t sh,
                                    int64_t ss, int T, int H, int W, int Hp, int Wp, int D,
                                    const uint8_t* __restrict__ valid,
                                    const uint16_t* __restrict__ norms, float* __restrict__ part,
                                    float* __restrict__ apart) {
  const int ZH = Hp / 8, ZW = Wp / 8;
  const int z = blockIdx.x >> 3, lt = blockIdx.x & 7;
  const int zt = z / (ZH * ZW), zh = (z / ZW) % ZH, zw = z % ZW;
  const int t = zt * 8 + lt;
  const int c0 = 2 * threadIdx.x;
  float* P = part + (int64_t)blockIdx.x * kPart * D;
  const float fheads = (float)heads;
  float cw0[8], cw1[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) cw0[i] = cw1[i] = 0.0f;
  float fr0 = 0.0f, fr1 = 0.0f;
  for (int lh = 0; lh < 8; ++lh) {
    float rh0 = 0.0f, rh1 = 0.0f;
    // the eight tokens of the row are independent until their ordered sums below:
    // their head sums run side by side (eight loads in flight per head step)
    const uint16_t* base[8];
    bool ok[8];
#pragma unroll
    for (int lw = 0; lw < 8; ++lw) {
      int64_t s = 0;
      ok[lw] = token_valid(t, zh * 8 + lh, zw * 8 + lw, T, H, W, Hp, Wp, valid, s);
      base[lw] = v + (ok[lw] ? s : 0) * ss + c0;
    }
    float a0[8], a1[8];
#pragma unroll
    for (int lw = 0; lw < 8; ++lw) a0[lw] = a1[lw] = 0.0f;
    for (int hh = 0; hh < heads; ++hh) {
      uint32_t u[8];
#pragma unroll
      for (int lw = 0; lw < 8; ++lw)
        u[lw] = ok[lw] ? __ldg(reinterpret_cast<const uint32_t*>(base[lw] + (int64_t)hh * sh)) : 0u;
#pragma unroll
      for (int lw = 0; lw < 8; ++lw) {
        a0[lw] = __fadd_rn(a0[lw], __uint_as_float(u[lw] << 16));
        a1[lw] = __fadd_rn(a1[lw], __uint_as_float(u[lw] & 0xffff0000u));
      }
    }
#pragma unroll
    for (int lw = 0; lw < 8; ++lw) {
      if (!ok[lw]) continue;
      const float x0 = __bfloat162float(__float2bfloat16_rn(__fdiv_rn(a0[lw], fheads)));
      const float x1 = __bfloat162float(__float2bfloat16_rn(__fdiv_rn(a1[lw], fheads)));
      rh0 = __fadd_rn(rh0, x0);
      rh1 = __fadd_rn(rh1, x1);
      cw0[lw] = __fadd_rn(cw0[lw], x0);
      cw1[lw] = __fadd_rn(cw1[lw], x1);
    }
    P[(1 + lh) * D + c0] = rh0;
    P[(1 + lh) * D + c0 + 1] = rh1;
    fr0 = __fadd_rn(fr0, rh0);
    fr1 = __fadd_rn(fr1, rh1);
  }
  P[c0] = fr0;
  P[c0 + 1] = fr1;
#pragma unroll
  for (int lw = 0; lw < 8; ++lw) {
    P[(9 + lw) * D + c0] = cw0[lw];
    P[(9 + lw) * D + c0 + 1] = cw1[lw];
  }
  if (threadIdx.x == 0) {
    float* A = apart + (int64_t)blockIdx.x * kPart;
    float cw[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float fr = 0.0f;
    for (int lh = 0; lh < 8; ++lh) {
      float rh = 0.0f;
      for (int lw = 0; lw < 8; ++lw) {
        int64_t s;
        if (!token_valid(t, zh * 8 + lh, zw * 8 + lw, T, H, W, Hp, Wp, valid, s)) continue;
        const float x = norms != nullptr ? bfbits2f(norms[s]) : 0.0f;
        rh = __fadd_rn(rh, x);
        cw[lw] = __fadd_rn(cw[lw], x);
      }
      A[1 + lh] = rh;
      fr = __fadd_rn(fr, rh);
    }
    A[0] = fr;
    for (int lw = 0; lw < 8; ++lw) A[9 + lw] = cw[lw];
  }
}

// The same partial sums with the eight rows of the frame in parallel (16 <= D <= 128): a
// CTA of 8 x D/2 threads (two CTAs per SM), thread (lh, channel pair) makes row lh's
// head means (kZoneHeads heads' loads in flight per step) and its row sums; the
// column sums over the rows and the frame sum are then taken from shared memory in
// row order lh = 0..7, so every sum has the summation order of zone_partial_kernel
// and the result is the same bit for bit.
constexpr int kZoneHeads = 2;
__global__ void __launch_bounds__(512, 2) zone_partial_rows_kernel(
    const uint16_t* __restrict__ v, int heads, int64_t sh, int64_t ss, int T, int H, int W, int Hp,
    int Wp, int D, const uint8_t* __restrict__ valid, const uint16_t* __restrict__ norms,
    float* __restrict__ part, float* __restrict__ apart) {
  extern __shared__ float zsm[];
  float* xs = zsm;           // [8 lh][8 lw][D] head means of the frame's tokens
  float* rs = zsm + 64 * D;  // [8 lh][D] row sums
  __shared__ float an[64];
  __shared__ unsigned long long okm;
  const int ZH = Hp / 8, ZW = Wp / 8;
  const int z = blockIdx.x >> 3, lt = blockIdx.x & 7;
  const int zt = z / (ZH * ZW), zh = (z / ZW) % ZH, zw = z % ZW;
  const int t = zt * 8 + lt;
  const int half = D / 2;
  const int lh = threadIdx.x / half;
  const int c0 = 2 * (threadIdx.x - lh * half);
  float* P = part + (int64_t)blockIdx.x * kPart * D;
  const float fheads = (float)heads;
  if (threadIdx.x == 0) okm = 0ull;
  __syncthreads();
  if (threadIdx.x < 64) {
    int64_t s = 0;
    const bool ok = token_valid(t, zh * 8 + threadIdx.x / 8, zw * 8 + threadIdx.x % 8, T, H, W, Hp, Wp,
                                valid, s);
    an[threadIdx.x] = ok && norms != nullptr ? bfbits2f(__ldg(norms + s)) : 0.0f;
    if (ok) atomicOr(&okm, 1ull << threadIdx.x);
  }
  // the row's eight tokens are consecutive source tokens (w = 8 zw + lw); only the
  // valid ones are loaded
  unsigned okb = 0;
#pragma unroll
  for (int lw = 0; lw < 8; ++lw) {
    int64_t s = 0;
    if (token_valid(t, zh * 8 + lh, zw * 8 + lw, T, H, W, Hp, Wp, valid, s)) okb |= 1u << lw;
  }
  const uint16_t* vb = v + (okb ? (((int64_t)t * H + zh * 8 + lh) * W + zw * 8) * ss + c0 : 0);
  float a0[8], a1[8];
#pragma unroll
  for (int lw = 0; lw < 8; ++lw) a0[lw] = a1[lw] = 0.0f;
  int hh = 0;
  // kZoneHeads heads' loads in flight per step, summed in head order
  for (; hh + kZoneHeads <= heads; hh += kZoneHeads) {
    uint32_t u[kZoneHeads][8];
#pragma unroll
    for (int e = 0; e < kZoneHeads; ++e)
#pragma unroll
      for (int lw = 0; lw < 8; ++lw)
        u[e][lw] = (okb >> lw) & 1u
                       ? __ldg(reinterpret_cast<const uint32_t*>(vb + lw * ss + (int64_t)(hh + e) * sh))
                       : 0u;
#pragma unroll
    for (int e = 0; e < kZoneHeads; ++e)
#pragma unroll
      for (int lw = 0; lw < 8; ++lw) {
        a0[lw] = __fadd_rn(a0[lw], __uint_as_float(u[e][lw] << 16));
        a1[lw] = __fadd_rn(a1[lw], __uint_as_float(u[e][lw] & 0xffff0000u));
      }
  }
  for (; hh < heads; ++hh) {
#pragma unroll
    for (int lw = 0; lw < 8; ++lw) {
      const uint32_t u =
          (okb >> lw) & 1u ? __ldg(reinterpret_cast<const uint32_t*>(vb + lw * ss + (int64_t)hh * sh)) : 0u;
      a0[lw] = __fadd_rn(a0[lw], __uint_as_float(u << 16));
      a1[lw] = __fadd_rn(a1[lw], __uint_as_float(u & 0xffff0000u));
    }
  }
  float rh0 = 0.0f, rh1 = 0.0f;
#pragma unroll
  for (int lw = 0; lw < 8; ++lw) {
    if (!((okb >> lw) & 1u)) continue;
    const float x0 = __bfloat162float(__float2bfloat16_rn(__fdiv_rn(a0[lw], fheads)));
    const float x1 = __bfloat162float(__float2bfloat16_rn(__fdiv_rn(a1[lw], fheads)));
    rh0 = __fadd_rn(rh0, x0);
    rh1 = __fadd_rn(rh1, x1);
    xs[(lh * 8 + lw) * D + c0] = x0;
    xs[(lh * 8 + lw) * D + c0 + 1] = x1;
  }
  P[(1 + lh) * D + c0] = rh0;
  P[(1 + lh) * D + c0 + 1] = rh1;
  rs[lh * D + c0] = rh0;
  rs[lh * D + c0 + 1] = rh1;
  __syncthreads();
  const unsigned long long m = okm;
  {
    // column lw = lh of the frame, summed over its rows in order
    const int lw = lh;
    float cw0 = 0.0f, cw1 = 0.0f;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      if (!((m >> (r * 8 + lw)) & 1ull)) continue;
      cw0 = __fadd_rn(cw0, xs[(r * 8 + lw) * D + c0]);
      cw1 = __fadd_rn(cw1, xs[(r * 8 + lw) * D + c0 + 1]);
    }
    P[(9 + lw) * D + c0] = cw0;
    P[(9 + lw) * D + c0 + 1] = cw1;
  }
  if (lh == 0) {
    float fr0 = 0.0f, fr1 = 0.0f;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      fr0 = __fadd_rn(fr0, rs[r * D + c0]);
      fr1 = __fadd_rn(fr1, rs[r * D + c0 + 1]);
    }
    P[c0] = fr0;
    P[c0 + 1] = fr1;
  }
  if (threadIdx.x == 0) {
    float* A = apart + (int64_t)blockIdx.x * kPart;
    float cw[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float fr = 0.0f;
    for (int r = 0; r < 8; ++r) {
      float rh = 0.0f;
      for (int lw = 0; lw < 8; ++lw) {
        if (!((m >> (r * 8 + lw)) & 1ull)) continue;
        const float x = an[r * 8 + lw];
        rh = __fadd_rn(rh, x);
        cw[lw] = __fadd_rn(cw[lw], x);
      }
      A[1 + r] = rh;
      fr = __fadd_rn(fr, rh);
    }
    A[0] = fr;
    for (int lw = 0; lw < 8; ++lw) A[9 + lw] = cw[lw];
  }
}

// Stage 2: one CTA per zone; combine the eight frames in order lt = 0..7.
__global__ void zone_combine_kernel(const float* __restrict__ part, const float* __restrict__ apart,
                                    int T, int H, int W, int Hp, int Wp, int D,
                                    const uint8_t* __restrict__ valid,
                                    float* __restrict__ packed, uint8_t* __restrict__ axis_valid,
                                    float* __restrict__ audio) {
  const int ZH = Hp / 8, ZW = Wp / 8;
  const int z = blockIdx.x;
  const int zt = z / (ZH * ZW), zh = (z / ZW) % ZH, zw = z % ZW;
  __shared__ int cT[8], cH[8], cW[8], call;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 8; ++i) cT[i] = cH[i] = cW[i] = 0;
    call = 0;
    for (int lt = 0; lt < 8; ++lt)
      for (int lh = 0; lh < 8; ++lh)
        for (int lw = 0; lw < 8; ++lw) {
          int64_t s;
          if (!token_valid(zt * 8 + lt, zh * 8 + lh, zw * 8 + lw, T, H, W, Hp, Wp, valid, s)) continue;
          cT[lt]++;
          cH[lh]++;
          cW[lw]++;
          call++;
        }
  }
  __syncthreads();
  const float* Pz = part + (int64_t)z * 8 * kPart * D;
  float* pk = packed + (int64_t)z * 25 * D;
  const float fall = (float)(call > 0 ? call : 1);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float cs = 0.0f;
    for (int lt = 0; lt < 8; ++lt) cs = __fadd_rn(cs, Pz[(lt * kPart) * D + d]);
    pk[d] = __fdiv_rn(cs, fall);
    for (int lt = 0; lt < 8; ++lt)
      pk[D + lt * D + d] = __fdiv_rn(Pz[(lt * kPart) * D + d], (float)(cT[lt] > 0 ? cT[lt] : 1));
    for (int p = 0; p < 8; ++p) {
      float sh = 0.0f, sw = 0.0f;
      for (int lt = 0; lt < 8; ++lt) {
        sh = __fadd_rn(sh, Pz[(lt * kPart + 1 + p) * D + d]);
        sw = __fadd_rn(sw, Pz[(lt * kPart + 9 + p) * D + d]);
      }
      pk[D + 8 * D + p * D + d] = __fdiv_rn(sh, (float)(cH[p] > 0 ? cH[p] : 1));
      pk[D + 16 * D + p * D + d] = __fdiv_rn(sw, (float)(cW[p] > 0 ? cW[p] : 1));
    }
  }
  if (threadIdx.x == 0) {
    uint8_t* av = axis_valid + (int64_t)z * 24;
    for (int p = 0; p < 8; ++p) {
      av[p] = cT[p] > 0;
      av[8 + p] = cH[p] > 0;
      av[16 + p] = cW[p] > 0;
    }
    const float* Az = apart + (int64_t)z * 8 * kPart;
    float* au = audio + (int64_t)z * 25;
    float cs = 0.0f;
    for (int lt = 0; lt < 8; ++lt) cs = __fadd_rn(cs, Az[lt * kPart]);
    au[0] = __fdiv_rn(cs, fall);
    for (int lt = 0; lt < 8; ++lt)
      au[1 + lt] = __fdiv_rn(Az[lt * kPart], (float)(cT[lt] > 0 ? cT[lt] : 1));
    for (int p = 0; p < 8; ++p) {
      float sh = 0.0f, sw = 0.0f;
      for (int lt = 0; lt < 8; ++lt) {
        sh = __fadd_rn(sh, Az[lt * kPart + 1 + p]);
        sw = __fadd_rn(sw, Az[lt * kPart + 9 + p]);
      }
      au[9 + p] = __fdiv_rn(sh, (float)(cH[p] > 0 ? cH[p] : 1));
      au[17 + p] = __fdiv_rn(sw, (float)(cW[p] > 0 ? cW[p] : 1));
    }
  }
}

// ================================================================ a4/a6/a7
__device__ float masked_var8_dev(const float* a, const uint8_t* valid) {
  float n = 0.0f;
  for (int p = 0; p < 8; ++p) n = __fadd_rn(n, valid[p] ? 1.0f : 0.0f);
  if (n < 1.0f) n = 1.0f;
  float s = 0.0f;
  for (int p = 0; p < 8; ++p)
    if (valid[p]) s = __fadd_rn(s, a[p]);
  const float mean = __fdiv_rn(s, n);
  float q = 0.0f;
  for (int p = 0; p < 8; ++p)
    if (valid[p]) {
      const float t = __fsub_rn(a[p], mean);
      q = __fadd_rn(q, __fmul_rn(t, t));
    }
  return __fdiv_rn(q, n);
}

__device__ float block_max_f(float v, float* red) {
  for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = l < nw ? red[l] : -INFINITY;
    for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (l == 0) red[0] = v;
  }
  __syncthreads();
  v = red[0];
  __syncthreads();
  return v;
}

// One CTA.  Per-zone intermediates in shared memory: rho_raw, aniso[3], abar,
// vhat[3]; then the per-warp channel-term rows of the statistics pass.
__global__ void __launch_bounds__(512) shape_select_kernel(const float* __restrict__ packed,
                                    const uint8_t* __restrict__ axis_valid,
                                    const float* __restrict__ audio, int has_audio, int Nz, int D,
                                    int method, float lambda_a, float tau_128, float lambda_128,
                                    int64_t* __restrict__ shape_ids, float* __restrict__ g_out,
                                    float* __restrict__ rho_out) {
  extern __shared__ float zsm[];
  float* rho_raw = zsm;
  float* aniso = zsm + Nz;
  float* vhat = zsm + 4 * Nz;
  float* abar = zsm + 7 * Nz;
  __shared__ float red[32];
  const float EPS = 1e-6f;
  float lmax_r = -INFINITY, lmax_a = -INFINITY;
  // One warp per zone.  The per-channel terms of every statistic are computed by the
  // lanes in parallel (each term with the same operations as a one-thread pass) and
  // staged in shared memory; each sum over the channels is then taken by one lane in
  // channel order, so every result is the same bit for bit as a sequential pass.
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  float* T = zsm + 8 * Nz + warp * 6 * D;  // [6][D]: channel means, temporal terms,
                                           // 3 axis terms, spatial terms
  for (int z = warp; z < Nz; z += nwarps) {
    const float* pk = packed + (int64_t)z * 25 * D;
    const uint8_t* av = axis_valid + (int64_t)z * 24;
    uint32_t vm = 0;  // bit i: av[i] (the same 24 bytes for every lane)
    for (int i = 0; i < 24; ++i) vm |= (av[i] ? 1u : 0u) << i;
    float npairs = 0.0f;
#pragma unroll
    for (int p = 0; p < 7; ++p) npairs = __fadd_rn(npairs, ((vm >> (p + 1)) & (vm >> p) & 1u) ? 1.0f : 0.0f);
    if (npairs < 1.0f) npairs = 1.0f;
    float nax[3];
#pragma unroll
    for (int ax = 0; ax < 3; ++ax) {
      float n = 0.0f;
#pragma unroll
      for (int p = 0; p < 8; ++p) n = __fadd_rn(n, ((vm >> (8 * ax + p)) & 1u) ? 1.0f : 0.0f);
      nax[ax] = n < 1.0f ? 1.0f : n;
    }
    for (int d = lane; d < D; d += 32) {
      // the channel's 25 packed values (row 0: zone mean, rows 1 + 8 ax + p: axis-ax
      // slice means) in registers, all loads in flight at once
      float x[25];
#pragma unroll
      for (int r = 0; r < 25; ++r) x[r] = pk[r * D + d];
      T[d] = x[0];
      float a = 0.0f;
#pragma unroll
      for (int p = 0; p < 7; ++p)
        if ((vm >> (p + 1)) & (vm >> p) & 1u) {
          const float t = __fsub_rn(x[2 + p], x[1 + p]);
          a = __fadd_rn(a, __fmul_rn(t, t));
        }
      T[D + d] = __fdiv_rn(a, npairs);
#pragma unroll
      for (int ax = 0; ax < 3; ++ax) {
        float sm = 0.0f;
#pragma unroll
        for (int p = 0; p < 8; ++p)
          if ((vm >> (8 * ax + p)) & 1u) sm = __fadd_rn(sm, x[1 + 8 * ax + p]);
        const float mean = __fdiv_rn(sm, nax[ax]);
        float q = 0.0f;
#pragma unroll
        for (int p = 0; p < 8; ++p)
          if ((vm >> (8 * ax + p)) & 1u) {
            const float t = __fsub_rn(x[1 + 8 * ax + p], mean);
            q = __fadd_rn(q, __fmul_rn(t, t));
          }
        T[(2 + ax) * D + d] = __fdiv_rn(q, nax[ax]);
      }
    }
    __syncwarp();
    float gcm = 0.0f;
    if (lane == 0) {
      float sum = 0.0f;
      for (int d = 0; d < D; ++d) sum = __fadd_rn(sum, T[d]);
      gcm = __fdiv_rn(sum, (float)D);
    }
    gcm = __shfl_sync(0xffffffffu, gcm, 0);
    for (int d = lane; d < D; d += 32) {
      const float t = __fsub_rn(T[d], gcm);
      T[5 * D + d] = __fmul_rn(t, t);
    }
    __syncwarp();
    // lane 0: spatial (row 5), lane 1: temporal (row 1), lanes 2-4: axes (rows 2-4)
    float chain = 0.0f;
    if (lane < 5) {
      const float* row = T + (lane == 0 ? 5 : lane) * D;
      for (int d = 0; d < D; ++d) chain = __fadd_rn(chain, row[d]);
      chain = __fdiv_rn(chain, (float)D);
    }
    const float temporal = __shfl_sync(0xffffffffu, chain, 1);
    const float vT = __shfl_sync(0xffffffffu, chain, 2);
    const float vH = __shfl_sync(0xffffffffu, chain, 3);
    const float vW = __shfl_sync(0xffffffffu, chain, 4);
    if (lane == 0) {
      const float spatial = chain;
      rho_raw[z] = __fadd_rn(spatial, temporal);
      float asum = __fadd_rn(__fadd_rn(vT, vH), vW);
      if (asum < EPS) asum = EPS;
      aniso[3 * z + 0] = __fdiv_rn(vT, asum);
      aniso[3 * z + 1] = __fdiv_rn(vH, asum);
      aniso[3 * z + 2] = __fdiv_rn(vW, asum);
      if (has_audio) {
        const float* au = audio + (int64_t)z * 25;
        abar[z] = au[0];
        const float aT = masked_var8_dev(au + 1, av);
        const float aH = masked_var8_dev(au + 9, av + 8);
        const float aW = masked_var8_dev(au + 17, av + 16);
        float den = __fadd_rn(__fadd_rn(aT, aH), aW);
        if (den < EPS) den = EPS;
        vhat[3 * z + 0] = __fdiv_rn(aT, den);
        vhat[3 * z + 1] = __fdiv_rn(aH, den);
        vhat[3 * z + 2] = __fdiv_rn(aW, den);
      } else {
        abar[z] = 0.0f;
        vhat[3 * z + 0] = vhat[3 * z + 1] = vhat[3 * z + 2] = 0.0f;
      }
      lmax_r = fmaxf(lmax_r, rho_raw[z]);
      lmax_a = fmaxf(lmax_a, abar[z]);
    }
    __syncwarp();
  }
  __syncthreads();
  float rmax = block_max_f(lmax_r, red);
  float amax = block_max_f(lmax_a, red);
  if (rmax < EPS) rmax = EPS;
  if (amax < EPS) amax = EPS;
  for (int z = threadIdx.x; z < Nz; z += blockDim.x) {
    const float rho = __fdiv_rn(rho_raw[z], rmax);
    const float an = has_audio ? __fdiv_rn(abar[z], amax) : 0.0f;
    const float la = __fmul_rn(lambda_a, an);
    float g[3];
    for (int d = 0; d < 3; ++d) {
      g[d] = __fadd_rn(aniso[3 * z + d], __fmul_rn(la, vhat[3 * z + d]));
      if (g[d] < 1e-4f) g[d] = 1e-4f;
    }
    if (g_out) {
      g_out[3 * z] = g[0];
      g_out[3 * z + 1] = g[1];
      g_out[3 * z + 2] = g[2];
    }
    if (rho_out) rho_out[z] = rho;
    const bool forbid128 = rho >= tau_128;
    int best = 0;
    float bestv = INFINITY;
    if (method == 0) {
      const float c23 = (float)(-2.0 / 3.0);
      float lr[3];
      for (int d = 0; d < 3; ++d) lr[d] = __fmul_rn(c23, det_log2f(g[d]));
      const float sum = __fadd_rn(__fadd_rn(lr[0], lr[1]), lr[2]);
      const float add = __fdiv_rn(__fsub_rn(6.0f, sum), 3.0f);
      const float li0 = __fadd_rn(lr[0], add), li1 = __fadd_rn(lr[1], add), li2 = __fadd_rn(lr[2], add);
      for (int c = 0; c < kNumShapes; ++c) {
        float dist;
        if (forbid128 && c >= kNumShapes64) {
          dist = INFINITY;
        } else {
          const float a0 = __fsub_rn((float)(31 - __clz(shape_dim(c, 0))), li0);
          const float a1 = __fsub_rn((float)(31 - __clz(shape_dim(c, 1))), li1);
          const float a2 = __fsub_rn((float)(31 - __clz(shape_dim(c, 2))), li2);
          dist = __fadd_rn(__fadd_rn(__fmul_rn(a0, a0), __fmul_rn(a1, a1)), __fmul_rn(a2, a2));
        }
        if (dist < bestv) {
          bestv = dist;
          best = c;
        }
      }
    } else {
      const float bonus = __fmul_rn(lambda_128, __fsub_rn(1.0f, rho));
      for (int c = 0; c < kNumShapes; ++c) {
        float pen;
        if (forbid128 && c >= kNumShapes64) {
          pen = INFINITY;
        } else {
          pen = __fadd_rn(__fadd_rn(__fmul_rn(g[0], (float)shape_dim(c, 0)),
                                    __fmul_rn(g[1], (float)shape_dim(c, 1))),
                          __fmul_rn(g[2], (float)shape_dim(c, 2)));
          pen = __fsub_rn(pen, __fmul_rn(bonus, c >= kNumShapes64 ? 1.0f : 0.0f));
        }
        if (pen < bestv) {
          bestv = pen;
          best = c;
        }
      }
    }
    shape_ids[z] = best;
  }
}

// ================================================================ a8/a9
// Rearranged row r of zone z (shape c) -> local flat lt*64 + lh*8 + lw.
// Inverse of dynamic_block_attention.py:41-51: r = blk*bsz + off with
// blk = (nt*Nh + nh)*Nw + nw, off = (it*bh + ih)*bw + iw.
__device__ __forceinline__ void local_coords(int c, int r, int& lt, int& lh, int& lw) {
  const int bt = shape_dim(c, 0), bh = shape_dim(c, 1), bw = shape_dim(c, 2);
  const int bsz = bt * bh * bw;
  const int Nh = 8 / bh, Nw = 8 / bw;
  const int blk = r / bsz, off = r % bsz;
  const int it = off / (bh * bw), ih = (off / bw) % bh, iw = off % bw;
  const int nt = blk / (Nh * Nw), nh = (blk / Nw) % Nh, nw = blk % Nw;
  lt = nt * bt + it;
  lh = nh * bh + ih;
  lw = nw * bw + iw;
}

// One CTA of 1024 threads: exclusive scan of blocks-per-zone, then tile maps.
__global__ void __launch_bounds__(1024) block_map_kernel(const int64_t* __restrict__ shape_ids, int Nz,
                                 int32_t* __restrict__ block_of_tile,
                                 int32_t* __restrict__ block_tiles, int32_t* __restrict__ n_blocks) {
  __shared__ int warp_sums[32];
  __shared__ int carry;
  const int n_tiles = Nz * 8;
  if (threadIdx.x == 0) carry = 0;
  // sentinel fill of every block row first
  for (int i = threadIdx.x; i < (n_tiles + 1) * 2; i += blockDim.x) block_tiles[i] = n_tiles;
  __syncthreads();
  for (int base = 0; base < Nz; base += blockDim.x) {
    const int z = base + threadIdx.x;
    int c = 0, nbz = 0;
    if (z < Nz) {
      c = (int)shape_ids[z];
      nbz = 512 / shape_tokens(c);
    }
    // block-wide exclusive scan of nbz
    int v = nbz;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    for (int o = 1; o < 32; o <<= 1) {
      int n = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += n;
    }
    if (lane == 31) warp_sums[w] = v;
    __syncthreads();
    if (w == 0) {
      int s = lane < (int)(blockDim.x >> 5) ? warp_sums[lane] : 0;
      for (int o = 1; o < 32; o <<= 1) {
        int n = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += n;
      }
      warp_sums[lane] = s;  // inclusive
    }
    __syncthreads();
    const int excl = carry + (w > 0 ? warp_sums[w - 1] : 0) + v - nbz;
    if (z < Nz) {
      const int tpb = shape_tokens(c) / 64;
      for (int tl = 0; tl < 8; ++tl) {
        const int j = z * 8 + tl;
        const int b = excl + tl / tpb;
        block_of_tile[j] = b;
        block_tiles[b * 2 + tl % tpb] = j;
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) carry += warp_sums[(blockDim.x >> 5) - 1];
    __syncthreads();
  }
  if (threadIdx.x == 0) *n_blocks = carry;
}

__global__ void perm_kernel(const int64_t* __restrict__ shape_ids, int Hp, int Wp, int64_t S,
                            int32_t* __restrict__ src_idx, int32_t* __restrict__ inv_idx) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= S) return;
  const int ZH = Hp / 8, ZW = Wp / 8;
  const int z = (int)(r >> 9), rr = (int)(r & 511);
  const int zt = z / (ZH * ZW), zh = (z / ZW) % ZH, zw = z % ZW;
  int lt, lh, lw;
  local_coords((int)shape_ids[z], rr, lt, lh, lw);
  const int64_t g = ((int64_t)(zt * 8 + lt) * Hp + (zh * 8 + lh)) * Wp + (zw * 8 + lw);
  src_idx[r] = (int32_t)g;
  inv_idx[g] = (int32_t)r;
}

// One warp per tile.
__device__ __forceinline__ bool padded_valid(int64_t g, int T, int H, int W, int Hp, int Wp,
                                             const uint8_t* __restrict__ valid) {
  const int t = (int)(g / ((int64_t)Hp * Wp));
  const int h = (int)((g / Wp) % Hp);
  const int w = (int)(g % Wp);
  if (t >= T || h >= H || w >= W) return false;
  return valid == nullptr || valid[g] != 0;
}

__global__ void tile_valid_kernel(const int32_t* __restrict__ src_idx,
                                  const uint8_t* __restrict__ valid, int64_t n_tiles, int T, int H,
                                  int W, int Hp, int Wp, uint64_t* __restrict__ tile_bits,
                                  int32_t* __restrict__ tile_count) {
  const int64_t j = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (j >= n_tiles) return;
  const bool v0 = padded_valid(src_idx[j * 64 + lane], T, H, W, Hp, Wp, valid);
  const bool v1 = padded_valid(src_idx[j * 64 + 32 + lane], T, H, W, Hp, Wp, valid);
  const uint32_t b0 = __ballot_sync(0xffffffffu, v0);
  const uint32_t b1 = __ballot_sync(0xffffffffu, v1);
  if (lane == 0) {
    tile_bits[j] = (uint64_t)b0 | ((uint64_t)b1 << 32);
    tile_count[j] = __popc(b0) + __popc(b1);
  }
}

// ================================================================ a10/a17
// 16-byte chunks; rows of D bf16.  Grid: (ceil(rows * chunks / 256), heads); the
// index arithmetic is 32-bit (rows * chunks < 2^31, checked by the entry points).
__global__ void gather_rows_kernel(const uint4* __restrict__ x, int64_t xsh, int64_t xss, int chunks,
                                   int T, int H, int W, int Hp, int Wp, int Sp,
                                   const int32_t* __restrict__ src_idx, uint4* __restrict__ out,
                                   int64_t osh) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= Sp * chunks) return;
  const int h = blockIdx.y;
  const int r = j / chunks, c = j - r * chunks;
  const int g = src_idx[r];
  const int hw = Hp * Wp;
  const int t = g / hw;
  const int rem = g - t * hw;
  const int hh = rem / Wp;
  const int w = rem - hh * Wp;
  uint4 val = make_uint4(0, 0, 0, 0);
  if (t < T && hh < H && w < W) {
    const int64_t s = ((int64_t)t * H + hh) * W + w;
    val = __ldg(x + ((int64_t)h * xsh + s * xss) / 8 + c);
  }
  out[((int64_t)h * osh) / 8 + (int64_t)j] = val;
}

// The same gathers with each thread moving one 16-byte chunk of kRowsPerThread
// rows (chunks | 256: the block covers 256 / chunks rows per pass): every load
// is issued before the first store, so a thread keeps 64 bytes in flight -- a
// one-chunk-per-thread copy holds too few bytes in flight to reach HBM rate.
constexpr int kRowsPerThread = 4;
__global__ void __launch_bounds__(256) gather_rows4_kernel(
    const uint4* __restrict__ x, int64_t xsh, int64_t xss, int chunks, int T, int H, int W, int Hp,
    int Wp, int Sp, const int32_t* __restrict__ src_idx, uint4* __restrict__ out, int64_t osh) {
  const int rpp = 256 / chunks;  // rows per pass
  const int c = threadIdx.x % chunks;
  const int r0 = blockIdx.x * (rpp * kRowsPerThread) + threadIdx.x / chunks;
  const int h = blockIdx.y;
  const int hw = Hp * Wp;
  const uint4* xh = x + ((int64_t)h * xsh) / 8 + c;
  uint4* oh = out + ((int64_t)h * osh) / 8 + c;
  uint4 val[kRowsPerThread];
#pragma unroll
  for (int u = 0; u < kRowsPerThread; ++u) {
    const int r = r0 + u * rpp;
    val[u] = make_uint4(0, 0, 0, 0);
    if (r < Sp) {
      const int g = __ldg(src_idx + r);
      const int t = g / hw;
      const int rem = g - t * hw;
      const int hh = rem / Wp;
      const int w = rem - hh * Wp;
      if (t < T && hh < H && w < W) val[u] = __ldg(xh + ((((int64_t)t * H + hh) * W + w) * xss) / 8);
    }
  }
#pragma unroll
  for (int u = 0; u < kRowsPerThread; ++u) {
    const int r = r0 + u * rpp;
    if (r < Sp) oh[(int64_t)r * chunks] = val[u];
  }
}

__global__ void __launch_bounds__(256) scatter_rows4_kernel(
    const uint4* __restrict__ x, int64_t xsh, int chunks, int T, int H, int W, int Hp, int Wp,
    const int32_t* __restrict__ inv_idx, uint4* __restrict__ out, int64_t osh, int64_t oss) {
  const int rpp = 256 / chunks;
  const int c = threadIdx.x % chunks;
  const int s0 = blockIdx.x * (rpp * kRowsPerThread) + threadIdx.x / chunks;
  const int h = blockIdx.y;
  const int S = T * H * W, hw = H * W;
  const uint4* xh = x + ((int64_t)h * xsh) / 8 + c;
  uint4* oh = out + ((int64_t)h * osh) / 8 + c;
  uint4 val[kRowsPerThread];
#pragma unroll
  for (int u = 0; u < kRowsPerThread; ++u) {
    const int sx = s0 + u * rpp;
    if (sx < S) {
      const int t = sx / hw;
      const int rem = sx - t * hw;
      const int hh = rem / W;
      const int w = rem - hh * W;
      const int r = __ldg(inv_idx + ((int64_t)t * Hp + hh) * Wp + w);
      val[u] = __ldg(xh + (int64_t)r * chunks);
    }
  }
#pragma unroll
  for (int u = 0; u < kRowsPerThread; ++u) {
    const int sx = s0 + u * rpp;
    if (sx < S) oh[((int64_t)sx * oss) / 8] = val[u];
  }
}

// Token-major forms, used when a token's heads lie side by side (head stride == D,
// the [S, H, D] layout of the model and of the Ulysses receive buffer): one CTA moves
// kTokRows tokens with every head, so each token's source (gather) or destination
// (scatter) is one contiguous heads*D*2-byte span instead of `heads` 256-byte pieces
// kilobytes apart, and each head's side is kTokRows consecutive tile-order rows.
// Consecutive threads take consecutive 16-byte chunks of that span; a thread issues
// kTokUnroll loads before its stores.
constexpr int kTokRows = 8;
constexpr int kTokUnroll = 4;
__global__ void __launch_bounds__(256) gather_rows_tok_kernel(
    const uint4* __restrict__ x, int64_t xss, int heads, int chunks, int T, int H, int W, int Hp,
    int Wp, int Sp, const int32_t* __restrict__ src_idx, uint4* __restrict__ out, int64_t osh) {
  __shared__ int64_t s_off[kTokRows];  // 16-byte offset of the token's span, -1 for padding
  const int r0 = blockIdx.x * kTokRows;
  if (threadIdx.x < kTokRows) {
    const int r = r0 + threadIdx.x;
    int64_t off = -1;
    if (r < Sp) {
      const int g = __ldg(src_idx + r);
      const int hw = Hp * Wp;
      const int t = g / hw;
      const int rem = g - t * hw;
      const int hh = rem / Wp;
      const int w = rem - hh * Wp;
      if (t < T && hh < H && w < W) off = ((((int64_t)t * H + hh) * W + w) * xss) / 8;
    }
    s_off[threadIdx.x] = off;
  }
  __syncthreads();
  const int per_row = heads * chunks;
  const int total = kTokRows * per_row;
  const int64_t osh16 = osh / 8;
  for (int i0 = threadIdx.x; i0 < total; i0 += 256 * kTokUnroll) {
    uint4 val[kTokUnroll];
#pragma unroll
    for (int u = 0; u < kTokUnroll; ++u) {
      const int i = i0 + u * 256;
      val[u] = make_uint4(0, 0, 0, 0);
      if (i < total) {
        const int row = i / per_row;
        const int64_t off = s_off[row];
        if (off >= 0) val[u] = __ldg(x + off + (i - row * per_row));
      }
    }
#pragma unroll
    for (int u = 0; u < kTokUnroll; ++u) {
      const int i = i0 + u * 256;
      if (i < total) {
        const int row = i / per_row;
        const int rem = i - row * per_row;
        const int h = rem / chunks;
        const int r = r0 + row;
        if (r < Sp) out[h * osh16 + (int64_t)r * chunks + (rem - h * chunks)] = val[u];
      }
    }
  }
}

__global__ void __launch_bounds__(256) scatter_rows_tok_kernel(
    const uint4* __restrict__ x, int64_t xsh, int heads, int chunks, int T, int H, int W, int Hp,
    int Wp, const int32_t* __restrict__ inv_idx, uint4* __restrict__ out, int64_t oss) {
  __shared__ int s_row[kTokRows];  // tile-order row of the token
  const int S = T * H * W;
  const int s0 = blockIdx.x * kTokRows;
  if (threadIdx.x < kTokRows) {
    const int s = s0 + threadIdx.x;
    int r = 0;
    if (s < S) {
      const int hw = H * W;
      const int t = s / hw;
      const int rem = s - t * hw;
      const int hh = rem / W;
      const int w = rem - hh * W;
      r = __ldg(inv_idx + ((int64_t)t * Hp + hh) * Wp + w);
    }
    s_row[threadIdx.x] = r;
  }
  __syncthreads();
  const int per_row = heads * chunks;
  const int total = kTokRows * per_row;
  const int64_t xsh16 = xsh / 8, oss16 = oss / 8;
  for (int i0 = threadIdx.x; i0 < total; i0 += 256 * kTokUnroll) {
    uint4 val[kTokUnroll];
#pragma unroll
    for (int u = 0; u < kTokUnroll; ++u) {
      const int i = i0 + u * 256;
      if (i < total) {
        const int row = i / per_row;
        const int rem = i - row * per_row;
        const int h = rem / chunks;
        val[u] = make_uint4(0, 0, 0, 0);
        if (s0 + row < S)
          val[u] = __ldg(x + h * xsh16 + (int64_t)s_row[row] * chunks + (rem - h * chunks));
      }
    }
#pragma unroll
    for (int u = 0; u < kTokUnroll; ++u) {
      const int i = i0 + u * 256;
      if (i < total) {
        const int row = i / per_row;
        if (s0 + row < S) out[(int64_t)(s0 + row) * oss16 + (i - row * per_row)] = val[u];
      }
    }
  }
}

// Strided block copy for the Ulysses exchange layouts: row r of block o, `chunks`
// 16-byte chunks long, from src + o * so + r * sr to dst + o * dso + r * dsr (strides
// in 16-byte units).  A CTA moves kCopyRows consecutive rows of one block; consecutive
// threads take consecutive chunks, kTokUnroll loads in flight before their stores.
constexpr int kCopyRows = 8;
__global__ void __launch_bounds__(256) copy_rows_kernel(const uint4* __restrict__ src, int64_t so, int64_t sr,
                                                        uint4* __restrict__ dst, int64_t dso, int64_t dsr,
                                                        int64_t n_rows, int chunks) {
  const int64_t o = blockIdx.y;
  const int64_t r0 = (int64_t)blockIdx.x * kCopyRows;
  const int rows = (int)min((int64_t)kCopyRows, n_rows - r0);
  const int total = rows * chunks;
  const uint4* s = src + o * so + r0 * sr;
  uint4* d = dst + o * dso + r0 * dsr;
  for (int i0 = threadIdx.x; i0 < total; i0 += 256 * kTokUnroll) {
    uint4 val[kTokUnroll];
#pragma unroll
    for (int u = 0; u < kTokUnroll; ++u) {
      const int i = i0 + u * 256;
      if (i < total) {
        const int row = i / chunks;
        val[u] = __ldg(s + row * sr + (i - row * chunks));
      }
    }
#pragma unroll
    for (int u = 0; u < kTokUnroll; ++u) {
      const int i = i0 + u * 256;
      if (i < total) {
        const int row = i / chunks;
        d[row * dsr + (i - row * chunks)] = val[u];
      }
    }
  }
}

__global__ void scatter_rows_kernel(const uint4* __restrict__ x, int64_t xsh, int chunks, int T, int H,
                                    int W, int Hp, int Wp, const int32_t* __restrict__ inv_idx,
                                    uint4* __restrict__ out, int64_t osh, int64_t oss) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  const int S = T * H * W;
  if (j >= S * chunks) return;
  const int h = blockIdx.y;
  const int s = j / chunks, c = j - s * chunks;
  const int hw = H * W;
  const int t = s / hw;
  const int rem = s - t * hw;
  const int hh = rem / W;
  const int w = rem - hh * W;
  const int64_t g = ((int64_t)t * Hp + hh) * Wp + w;
  const int64_t r = inv_idx[g];
  out[((int64_t)h * osh + (int64_t)s * oss) / 8 + c] = __ldg(x + ((int64_t)h * xsh + r * chunks * 8) / 8 + c);
}

// ================================================================ a11
// One CTA per (block b, head h), D threads.  tile mean = sequential masked sum
// over the 64 rows / max(count, 1); block mean = ((0 + m0*c0) + m1*c1) / max(c, 1).
__global__ void pool_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ k, int64_t S,
                            int D, const int32_t* __restrict__ block_tiles,
                            const int32_t* __restrict__ n_blocks,
                            const uint64_t* __restrict__ tile_bits, float* __restrict__ qc,
                            float* __restrict__ kc, uint8_t* __restrict__ bvalid, int nb_max) {
  const int b = blockIdx.x, h = blockIdx.y;
  if (b >= *n_blocks) return;
  const int64_t n_tiles = S / 64;
  const int d = threadIdx.x;
  float oq = 0.0f, ok = 0.0f, cnt = 0.0f;
  for (int p = 0; p < 2; ++p) {
    const int j = block_tiles[2 * b + p];
    if (j >= n_tiles) continue;
    const uint64_t bits = tile_bits[j];
    const int c = __popcll(bits);
    const uint16_t* qr = q + ((int64_t)h * S + (int64_t)j * 64) * D + d;
    const uint16_t* kr = k + ((int64_t)h * S + (int64_t)j * 64) * D + d;
    float sq = 0.0f, sk = 0.0f;
    // sixteen rows' loads in flight (every row of the tile is in bounds), then the
    // masked sums in row order
    for (int i0 = 0; i0 < 64; i0 += 16) {
      uint16_t uq[16], uk[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        uq[i] = __ldg(qr + (int64_t)(i0 + i) * D);
        uk[i] = __ldg(kr + (int64_t)(i0 + i) * D);
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        if (!((bits >> (i0 + i)) & 1ull)) continue;
        sq = __fadd_rn(sq, bfbits2f(uq[i]));
        sk = __fadd_rn(sk, bfbits2f(uk[i]));
      }
    }
    const float fc = (float)c;
    const float den = c > 0 ? fc : 1.0f;
    oq = __fadd_rn(oq, __fmul_rn(__fdiv_rn(sq, den), fc));
    ok = __fadd_rn(ok, __fmul_rn(__fdiv_rn(sk, den), fc));
    cnt = __fadd_rn(cnt, fc);
  }
  const float den = cnt < 1.0f ? 1.0f : cnt;
  qc[((int64_t)h * nb_max + b) * D + d] = __fdiv_rn(oq, den);
  kc[((int64_t)h * nb_max + b) * D + d] = __fdiv_rn(ok, den);
  if (h == 0 && d == 0) bvalid[b] = cnt > 0.0f;
}

// The same pooling with two channels per thread (D/2 threads, 4-byte loads): each
// thread keeps 16 rows x 2 tensors x 4 bytes in flight; per channel the masked sums
// run in row order as above, so the means are the same bit for bit.
__global__ void pool2_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ k, int64_t S,
                             int D, const int32_t* __restrict__ block_tiles,
                             const int32_t* __restrict__ n_blocks,
                             const uint64_t* __restrict__ tile_bits, float* __restrict__ qc,
                             float* __restrict__ kc, uint8_t* __restrict__ bvalid, int nb_max) {
  const int b = blockIdx.x, h = blockIdx.y;
  if (b >= *n_blocks) return;
  const int64_t n_tiles = S / 64;
  const int d = 2 * threadIdx.x;
  float oq0 = 0.0f, oq1 = 0.0f, ok0 = 0.0f, ok1 = 0.0f, cnt = 0.0f;
  for (int p = 0; p < 2; ++p) {
    const int j = block_tiles[2 * b + p];
    if (j >= n_tiles) continue;
    const uint64_t bits = tile_bits[j];
    const int c = __popcll(bits);
    const uint32_t* qr = reinterpret_cast<const uint32_t*>(q + ((int64_t)h * S + (int64_t)j * 64) * D + d);
    const uint32_t* kr = reinterpret_cast<const uint32_t*>(k + ((int64_t)h * S + (int64_t)j * 64) * D + d);
    const int rs = D / 2;  // row stride in 4-byte words
    float sq0 = 0.0f, sq1 = 0.0f, sk0 = 0.0f, sk1 = 0.0f;
    for (int i0 = 0; i0 < 64; i0 += 16) {
      uint32_t uq[16], uk[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        uq[i] = __ldg(qr + (int64_t)(i0 + i) * rs);
        uk[i] = __ldg(kr + (int64_t)(i0 + i) * rs);
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        if (!((bits >> (i0 + i)) & 1ull)) continue;
        sq0 = __fadd_rn(sq0, __uint_as_float(uq[i] << 16));
        sq1 = __fadd_rn(sq1, __uint_as_float(uq[i] & 0xffff0000u));
        sk0 = __fadd_rn(sk0, __uint_as_float(uk[i] << 16));
        sk1 = __fadd_rn(sk1, __uint_as_float(uk[i] & 0xffff0000u));
      }
    }
    const float fc = (float)c;
    const float den = c > 0 ? fc : 1.0f;
    oq0 = __fadd_rn(oq0, __fmul_rn(__fdiv_rn(sq0, den), fc));
    oq1 = __fadd_rn(oq1, __fmul_rn(__fdiv_rn(sq1, den), fc));
    ok0 = __fadd_rn(ok0, __fmul_rn(__fdiv_rn(sk0, den), fc));
    ok1 = __fadd_rn(ok1, __fmul_rn(__fdiv_rn(sk1, den), fc));
    cnt = __fadd_rn(cnt, fc);
  }
  const float den = cnt < 1.0f ? 1.0f : cnt;
  float2* qo = reinterpret_cast<float2*>(qc + ((int64_t)h * nb_max + b) * D + d);
  float2* ko = reinterpret_cast<float2*>(kc + ((int64_t)h * nb_max + b) * D + d);
  *qo = make_float2(__fdiv_rn(oq0, den), __fdiv_rn(oq1, den));
  *ko = make_float2(__fdiv_rn(ok0, den), __fdiv_rn(ok1, den));
  if (h == 0 && d == 0) bvalid[b] = cnt > 0.0f;
}

// ================================================================ a12
// Register-tiled fp32 GEMM: score[a][b] = fma-chain over d = 0..D-1 of
// qc[a][d] * kc[b][d] (each accumulator updated once per d, in order).
// Per head: qc [na_max, D], kc [nb_max, D], score [na_max, nb_max].  The live
// sizes are *n_blocks x *n_blocks when n_blocks is given (dynamic layouts,
// known on the device only), else na_max x nb_max.  col_scale (nullable) multiplies
// column b's scores by col_scale[b] (score * score_modifier, bsa_interface.py:626-627).
constexpr int kScoreTile = 64;
__global__ void __launch_bounds__(256) score_kernel(const float* __restrict__ qc,
                                                    const float* __restrict__ kc, int D,
                                                    const int32_t* __restrict__ n_blocks,
                                                    int na_max, int nb_max,
                                                    const float* __restrict__ col_scale,
                                                    float* __restrict__ score) {
  extern __shared__ float ssm[];
  const int na = n_blocks ? *n_blocks : na_max;
  const int nb = n_blocks ? *n_blocks : nb_max;
  const int a0 = blockIdx.y * kScoreTile, b0 = blockIdx.x * kScoreTile, h = blockIdx.z;
  if (a0 >= na || b0 >= nb) return;
  float* Qs = ssm;                       // [D][64+4]
  float* Ks = ssm + D * (kScoreTile + 4);
  const float* qh = qc + (int64_t)h * na_max * D;
  const float* kh = kc + (int64_t)h * nb_max * D;
  for (int i = threadIdx.x; i < kScoreTile * D; i += blockDim.x) {
    const int r = i / D, d = i % D;
    Qs[d * (kScoreTile + 4) + r] = (a0 + r < na) ? qh[(int64_t)(a0 + r) * D + d] : 0.0f;
    Ks[d * (kScoreTile + 4) + r] = (b0 + r < nb) ? kh[(int64_t)(b0 + r) * D + d] : 0.0f;
  }
  __syncthreads();
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
  for (int d = 0; d < D; ++d) {
    float av[4], bv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) av[i] = Qs[d * (kScoreTile + 4) + ty * 4 + i];
#pragma unroll
    for (int j = 0; j < 4; ++j) bv[j] = Ks[d * (kScoreTile + 4) + tx * 4 + j];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = __fmaf_rn(av[i], bv[j], acc[i][j]);
  }
  float* sh = score + (int64_t)h * na_max * nb_max;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int a = a0 + ty * 4 + i;
    if (a >= na) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int b = b0 + tx * 4 + j;
      if (b < nb)
        sh[(int64_t)a * nb_max + b] = col_scale ? __fmul_rn(acc[i][j], col_scale[b]) : acc[i][j];
    }
  }
}

// ================================================================ a13/a14
// One CTA per (q block a, head h).  Keys are 32-bit patterns that order like
// the values: non-negative softmax weights as raw float bits (modes 0/1), raw
// scores mapped to an order-preserving unsigned integer (mode 2).
// Block -> tile maps: with block_tiles (dynamic layouts) block b covers the
// tiles block_tiles[2b], block_tiles[2b+1] (n_tiles = none); without it q block
// a covers tiles [a*tq, a*tq+tq) and key block b tiles [b*tk, b*tk+tk)
// (uniform chunks).  bvalid == nullptr means every key block is eligible.
constexpr int kSelThreads = 256;

__device__ __forceinline__ uint32_t f2key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ unsigned long long fix63(uint32_t wbits) {
  return __float2ull_rz(__fmul_rn(__uint_as_float(wbits), 0x1p63f));
}
__device__ __forceinline__ float round63(unsigned long long s) {
  return __fmul_rn(__ull2float_rn(s), 0x1p-63f);
}

template <typename T>
__device__ T block_sum_u64(T v, unsigned long long* red) {
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = l < nw ? (T)red[l] : (T)0;
    for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (l == 0) red[0] = v;
  }
  __syncthreads();
  v = (T)red[0];
  __syncthreads();
  return v;
}

// Warp 0 walks 256 buckets from high to low: lane l owns buckets 255-8l .. 248-8l.
// Returns (via shared state) the bucket where the running count (mode_mass=0)
// reaches `target_cnt`, or where the running mass rounds to >= pf (mode_mass=1).
struct RadixState {
  uint32_t prefix, pmask;
  int cnt_above;
  unsigned long long mass_above;
  int found;       // bucket found in this pass
  int bucket_cnt;  // count in the chosen bucket
};

__device__ void radix_walk(const uint32_t* hist_cnt, const unsigned long long* hist_mass, int shift,
                           int mode_mass, int target_cnt, float pf, RadixState* st) {
  const int lane = threadIdx.x & 31;
  int c8[8];
  unsigned long long m8[8];
  int lc = 0;
  unsigned long long lm = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int b = 255 - 8 * lane - i;
    c8[i] = hist_cnt[b];
    m8[i] = mode_mass ? hist_mass[b] : 0ull;
    lc += c8[i];
    lm += m8[i];
  }
  // inclusive scans across lanes (lane order == descending bucket order)
  int ic = lc;
  unsigned long long im = lm;
  for (int o = 1; o < 32; o <<= 1) {
    const int nc = __shfl_up_sync(0xffffffffu, ic, o);
    const unsigned long long nm = __shfl_up_sync(0xffffffffu, im, o);
    if (lane >= o) {
      ic += nc;
      im += nm;
    }
  }
  const int base_c = st->cnt_above;
  const unsigned long long base_m = st->mass_above;
  bool hit;
  if (mode_mass) hit = round63(base_m + im) >= pf;
  else hit = base_c + ic >= target_cnt;
  const uint32_t ball = __ballot_sync(0xffffffffu, hit);
  if (ball == 0) {
    if (lane == 0) st->found = 0;
    __syncwarp();
    return;
  }
  const int L = __ffs(ball) - 1;
  if (lane == L) {
    int c = base_c + ic - lc;
    unsigned long long m = base_m + im - lm;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const bool h2 = mode_mass ? (round63(m + m8[i]) >= pf) : (c + c8[i] >= target_cnt);
      if (h2) {
        const int b = 255 - 8 * lane - i;
        st->prefix |= (uint32_t)b << shift;
        st->pmask |= 0xffu << shift;
        st->cnt_above = c;
        st->mass_above = m;
        st->bucket_cnt = c8[i];
        st->found = 1;
        break;
      }
      c += c8[i];
      m += m8[i];
    }
  }
  __syncwarp();
}

// Histogram update aggregated per warp: lanes holding the same bucket add their
// count (and fixed-point mass) through one leader.  The keys of one radix pass
// concentrate in few buckets (probabilities share exponent bytes), so per-lane
// shared atomics would serialise on them; sums are integers, so the result is the
// same in any order.  Called by every lane of the warp (active = lane has a key).
__device__ __forceinline__ void hist_add_warp(uint32_t* hist_cnt, unsigned long long* hist_mass,
                                              bool active, int bkt, unsigned long long mass,
                                              bool with_mass) {
  const int lane = threadIdx.x & 31;
  const unsigned peers = __match_any_sync(0xffffffffu, active ? bkt : -1 - lane);
  unsigned long long sum = 0;
  if (with_mass) {
#pragma unroll 4
    for (int src = 0; src < 32; ++src) {
      const unsigned long long v = __shfl_sync(0xffffffffu, mass, src);
      if ((peers >> src) & 1u) sum += v;
    }
  }
  if (active && lane == __ffs(peers) - 1) {
    atomicAdd(&hist_cnt[bkt], (uint32_t)__popc(peers));
    if (with_mass) atomicAdd(&hist_mass[bkt], sum);
  }
}

__global__ void __launch_bounds__(kSelThreads) select_kernel(
    const float* __restrict__ score, const uint8_t* __restrict__ bvalid,
    const int32_t* __restrict__ n_blocks, int na_max, int nb_max,
    const int32_t* __restrict__ block_tiles, int tq, int tk,
    const uint64_t* __restrict__ tile_bits, int64_t n_qt, int64_t n_kt, int wq, int mode,
    double sparsity, double cdf, float sm_scale, uint32_t* __restrict__ bits_q) {
  // dynamic shared memory: fixed-point masses [nb_max] (u64, modes 0 / 1), keys
  // [nb_max], row bitmap [wq]
  extern __shared__ unsigned long long smem_u64[];
  unsigned long long* mass = smem_u64;
  uint32_t* keys = reinterpret_cast<uint32_t*>(smem_u64 + (mode == 2 ? 0 : nb_max));
  uint32_t* row = keys + nb_max;
  __shared__ uint32_t hist_cnt[256];
  __shared__ unsigned long long hist_mass[256];
  __shared__ unsigned long long hist_mass_w[kSelThreads / 32][256];  // per-warp mass histograms
  __shared__ unsigned long long red[32];
  __shared__ float redf[32];
  __shared__ RadixState st;
  __shared__ int tie_base[kSelThreads];
  const int na = n_blocks ? *n_blocks : na_max;
  const int nb = n_blocks ? *n_blocks : nb_max;
  const int a = blockIdx.x, h = blockIdx.y;
  if (a >= na) return;
  const float* srow = score + ((int64_t)h * na_max + a) * nb_max;
  const int tid = threadIdx.x;

  // selection sizes (computed in double exactly as Python does on the host)
  long long k_topk, ub;
  if (mode == 0) {
    k_topk = (long long)((1.0 - sparsity) * (double)nb);
    if (k_topk < 1) k_topk = 1;
    long long u = (long long)(cdf * (double)nb) + 1;
    ub = k_topk > u ? k_topk : u;
    if (ub > nb) ub = nb;
  } else if (mode == 1) {
    k_topk = 1;
    ub = (long long)(cdf * (double)nb) + 1;
    if (ub > nb) ub = nb;
  } else {
    k_topk = (long long)((1.0 - sparsity) * (double)nb);
    ub = nb;
  }
  const float pf = (float)cdf;
  long long n_eff = 0;
  uint32_t vstar = 0;  // the n_eff-th largest key
  int need = 0;        // how many keys equal to vstar are taken (lowest indices first)
  bool have_threshold = false;

  // Count passes: st.prefix <- the target-th largest key, st.cnt_above <- the number
  // of keys above it (4 byte-wise radix passes over the order-preserving keys).
  auto count_select = [&](long long target) {
    if (tid == 0) {
      st.prefix = 0;
      st.pmask = 0;
      st.cnt_above = 0;
      st.mass_above = 0;
      st.found = 1;
    }
    __syncthreads();
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      for (int i = tid; i < 256; i += blockDim.x) hist_cnt[i] = 0;
      __syncthreads();
      const uint32_t prefix = st.prefix, pmask = st.pmask;
      for (int i0 = 0; i0 < nb; i0 += blockDim.x) {  // warp-uniform trip count
        const int i = i0 + tid;
        const uint32_t kk = i < nb ? keys[i] : 0u;
        hist_add_warp(hist_cnt, hist_mass, i < nb && (kk & pmask) == prefix, (kk >> shift) & 0xff,
                      0ull, false);
      }
      __syncthreads();
      if (tid < 32) radix_walk(hist_cnt, hist_mass, shift, 0, (int)target, pf, &st);
      __syncthreads();
    }
  };

  if (mode == 2) {
    for (int i = tid; i < nb; i += blockDim.x)
      keys[i] = f2key((!bvalid || bvalid[i]) ? srow[i] : -INFINITY);
    n_eff = k_topk;
    __syncthreads();
  } else {
    float lmax = -INFINITY;
    for (int i = tid; i < nb; i += blockDim.x) {
      const float x = (!bvalid || bvalid[i]) ? __fmul_rn(srow[i], sm_scale) : -INFINITY;
      keys[i] = __float_as_uint(x);
      lmax = fmaxf(lmax, x);
    }
    const float mx = block_max_f(lmax, redf);
    unsigned long long lz = 0;
    for (int i = tid; i < nb; i += blockDim.x) {
      const float e = det_expf(__fsub_rn(__uint_as_float(keys[i]), mx));
      keys[i] = __float_as_uint(e);
      lz += __float2ull_rz(__fmul_rn(e, 0x1p50f));
    }
    const unsigned long long Z = block_sum_u64<unsigned long long>(lz, red);
    const float Zf = __fmul_rn(__ull2float_rn(Z), 0x1p-50f);
    for (int i = tid; i < nb; i += blockDim.x)
    {
      const uint32_t kk = __float_as_uint(__fdiv_rn(__uint_as_float(keys[i]), Zf));
      keys[i] = kk;
      mass[i] = fix63(kk);  // one conversion per key, reused by every mass pass
    }
    __syncthreads();
    // With S(m) the (fixed-point) mass of the m largest keys, the crossing point is
    // m_c = min{m : round(S(m)) >= pf} and n_eff = min(max(m_c, k_topk), ub)
    // (m_c - 1 clamped to ub first).  S is monotone, so round(S(k_topk)) >= pf means
    // m_c <= k_topk and n_eff = k_topk: when the top-k term is likely to dominate
    // (mode 0 with a small mass threshold) that is tested first, with the k_topk-th
    // key found by count passes, and the mass passes are skipped when it holds.
    // Both orders give the same n_eff, threshold and tie count.
    if (mode == 0 && cdf < 0.5) {
      count_select(k_topk);
      const uint32_t vk = st.prefix;
      const long long ca = st.cnt_above;
      unsigned long long part = 0;
      for (int i = tid; i < nb; i += blockDim.x)
        if (keys[i] > vk) part += mass[i];
      const unsigned long long Sk =
          block_sum_u64<unsigned long long>(part, red) + (unsigned long long)(k_topk - ca) * fix63(vk);
      if (round63(Sk) >= pf) {
        n_eff = k_topk;
        vstar = vk;
        need = (int)(k_topk - ca);
        have_threshold = true;
      }
      __syncthreads();
    }
    if (!have_threshold) {
      // crossing point m_c by mass radix descent
      if (tid == 0) {
        st.prefix = 0;
        st.pmask = 0;
        st.cnt_above = 0;
        st.mass_above = 0;
        st.found = 1;
        st.bucket_cnt = 0;
      }
      __syncthreads();
      bool crossed = true;
      for (int pass = 0; pass < 4 && crossed; ++pass) {
        const int shift = 24 - 8 * pass;
        for (int i = tid; i < 256; i += blockDim.x) hist_cnt[i] = 0;
        for (int i = tid; i < (kSelThreads / 32) * 256; i += blockDim.x) (&hist_mass_w[0][0])[i] = 0;
        __syncthreads();
        const uint32_t prefix = st.prefix, pmask = st.pmask;
        unsigned long long* wmass = hist_mass_w[tid >> 5];
        for (int i0 = 0; i0 < nb; i0 += blockDim.x) {  // warp-uniform trip count
          const int i = i0 + tid;
          const uint32_t kk = i < nb ? keys[i] : 0u;
          const bool in = i < nb && (kk & pmask) == prefix;
          hist_add_warp(hist_cnt, nullptr, in, (kk >> shift) & 0xff, 0ull, false);
          if (in) atomicAdd(&wmass[(kk >> shift) & 0xff], mass[i]);
        }
        __syncthreads();
        for (int i = tid; i < 256; i += blockDim.x) {
          unsigned long long m = 0;
#pragma unroll
          for (int w = 0; w < kSelThreads / 32; ++w) m += hist_mass_w[w][i];
          hist_mass[i] = m;
        }
        __syncthreads();
        if (tid < 32) radix_walk(hist_cnt, hist_mass, shift, 1, 0, pf, &st);
        __syncthreads();
        crossed = st.found != 0;
      }
      long long cnt_lt, m_c = 0, lo = 0;
      if (!crossed) {
        cnt_lt = ub;
      } else {
        // all remaining candidates share the value st.prefix; find j* in [1, bucket_cnt]
        const unsigned long long fv = fix63(st.prefix);
        long long hi = st.bucket_cnt;
        lo = 1;
        while (lo < hi) {
          const long long mid = (lo + hi) >> 1;
          if (round63(st.mass_above + (unsigned long long)mid * fv) >= pf) hi = mid;
          else lo = mid + 1;
        }
        m_c = st.cnt_above + lo;
        cnt_lt = m_c - 1 < ub ? m_c - 1 : ub;
      }
      long long n = cnt_lt + 1;
      if (n < k_topk) n = k_topk;
      if (n > nb) n = nb;
      n_eff = n < ub ? n : ub;
      if (crossed && n_eff == m_c) {
        // the n_eff-th largest key is the crossing key itself: st.prefix, with
        // st.cnt_above keys above it and lo of its ties taken
        vstar = st.prefix;
        need = (int)lo;
        have_threshold = true;
      }
      __syncthreads();
    }
  }

  // threshold element: the n_eff-th largest key (ties by lower index)
  for (int i = tid; i < wq; i += blockDim.x) row[i] = 0;
  if (n_eff > 0 && !have_threshold) {
    count_select(n_eff);
    vstar = st.prefix;
    need = (int)n_eff - st.cnt_above;
  }
  __syncthreads();
  // compaction: key > v*, or key == v* among the first `need` ties in index order
  if (n_eff > 0) {
    const int chunk = (nb + blockDim.x - 1) / blockDim.x;
    const int i0 = tid * chunk, i1 = min(nb, i0 + chunk);
    int nt = 0;
    for (int i = i0; i < i1; ++i) nt += keys[i] == vstar;
    // exclusive scan of nt over threads
    tie_base[tid] = nt;
    __syncthreads();
    if (tid == 0) {
      int run = 0;
      for (int i = 0; i < (int)blockDim.x; ++i) {
        const int x = tie_base[i];
        tie_base[i] = run;
        run += x;
      }
    }
    __syncthreads();
    int rank = tie_base[tid];
    for (int i = i0; i < i1; ++i) {
      const uint32_t kk = keys[i];
      bool sel = kk > vstar;
      if (kk == vstar) {
        sel = rank < need;
        ++rank;
      }
      if (!sel) continue;
      const int np = block_tiles ? 2 : tk;
      for (int p = 0; p < np; ++p) {
        const int kt = block_tiles ? block_tiles[2 * i + p] : i * tk + p;
        if (kt >= n_kt || tile_bits[kt] == 0ull) continue;
        atomicOr(&row[kt >> 5], 1u << (kt & 31));
      }
    }
  }
  __syncthreads();
  const int nq = block_tiles ? 2 : tq;
  for (int p = 0; p < nq; ++p) {
    const int qt = block_tiles ? block_tiles[2 * a + p] : a * tq + p;
    if (qt >= n_qt) continue;
    uint32_t* dst = bits_q + ((int64_t)h * n_qt + qt) * wq;
    for (int i = tid; i < wq; i += blockDim.x) dst[i] = row[i];
  }
}

// bits_k = transpose of bits_q per head, by 32x32 bit blocks (warp ballots):
// bits_q [n_qt][wk] (wk = ceil(n_kt / 32)) -> bits_k [n_kt][wq] (wq = ceil(n_qt / 32)).
__global__ void transpose_bits_kernel(const uint32_t* __restrict__ bq, int64_t n_qt, int64_t n_kt,
                                      int wq, int wk, uint32_t* __restrict__ bk) {
  const int bi = blockIdx.x;  // q-tile word block
  const int bj = blockIdx.y;  // k-tile word block
  const int h = blockIdx.z;
  const int lane = threadIdx.x;
  const int64_t qt = (int64_t)bi * 32 + lane;
  const uint32_t w = qt < n_qt ? bq[((int64_t)h * n_qt + qt) * wk + bj] : 0u;
  for (int b = 0; b < 32; ++b) {
    const uint32_t col = __ballot_sync(0xffffffffu, (w >> b) & 1u);
    const int64_t kt = (int64_t)bj * 32 + b;
    if (lane == 0 && kt < n_kt) bk[((int64_t)h * n_kt + kt) * wq + bi] = col;
  }
}

// ============================================================ uniform chunks
// rearrange_THW_to_3d_block order (bsa_interface.py:1105-1109): position
// p = ((((nt*Nh + nh)*Nw + nw)*ct + t)*ch + h)*cw + w holds the token at
// (nt*ct + t, nh*ch + h, nw*cw + w) of the padded grid.  Positions p >= Sp
// (rows that round the sequence up to whole tile pairs) get the sentinel Sp,
// which the gather reads as a zero row and the validity as padding.
__global__ void uniform_perm_kernel(int Hp, int Wp, int ct, int ch, int cw, int64_t Sp,
                                    int64_t n_rows, int32_t* __restrict__ src_idx,
                                    int32_t* __restrict__ inv_idx) {
  const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= n_rows) return;
  if (p >= Sp) {
    src_idx[p] = (int32_t)Sp;
    return;
  }
  const int Nh = Hp / ch, Nw = Wp / cw;
  int64_t r = p;
  const int w = (int)(r % cw);
  r /= cw;
  const int h = (int)(r % ch);
  r /= ch;
  const int t = (int)(r % ct);
  r /= ct;
  const int nw = (int)(r % Nw);
  r /= Nw;
  const int nh = (int)(r % Nh);
  const int64_t nt = r / Nh;
  const int64_t g = ((nt * ct + t) * Hp + (int64_t)nh * ch + h) * Wp + (int64_t)nw * cw + w;
  src_idx[p] = (int32_t)g;
  inv_idx[g] = (int32_t)p;
}

// masked_mean_pooling_compression / mean_pooling_compression
// (bsa_interface.py:164-201) over chunks of consecutive rows: per channel a
// sequential fp32 sum over the chunk's valid rows (bit s of the validity words;
// nullptr = all rows valid), divided by max(count, 1).  blockIdx.z picks x0 (S0
// rows per head, n0 chunks of chunk0 rows, validity bits0 -> out0) or x1 (S1, n1,
// chunk1, bits1 -> out1).  A thread owns 8 channels of one chunk (16-byte loads);
// a CTA of kPoolThreads threads covers kPoolThreads / (D / 8) chunks of a head.
// weights1 (nullable) replaces x1's validity by per-row weights w (Path B of the
// audio-guided path, audio_weighted_mean_pooling_compression, bsa_interface.py:
// 902-970): sum of the rounded products x * w divided by max(sum of w, 1).
constexpr int kPoolThreads = 128;
__global__ void __launch_bounds__(kPoolThreads) pool_chunk_kernel(
    const uint16_t* __restrict__ x0, const uint16_t* __restrict__ x1, int64_t S0, int64_t S1, int D,
    int chunk0, int n0, int chunk1, int n1, const uint64_t* __restrict__ bits0,
    const uint64_t* __restrict__ bits1, const float* __restrict__ weights1, float* __restrict__ out0,
    float* __restrict__ out1) {
  const int h = blockIdx.y, which = blockIdx.z;
  const int g8 = D / 8;                       // threads per chunk
  const int c = blockIdx.x * (kPoolThreads / g8) + threadIdx.x / g8;
  const int dg = (threadIdx.x % g8) * 8;      // first channel of this thread
  const int chunk = which ? chunk1 : chunk0;
  const int n = which ? n1 : n0;
  if (threadIdx.x >= (kPoolThreads / g8) * g8 || c >= n) return;
  const int64_t base = (int64_t)c * chunk;
  const uint4* x = reinterpret_cast<const uint4*>((which ? x1 : x0) +
                                                  ((int64_t)h * (which ? S1 : S0) + base) * D + dg);
  const int64_t rs = D / 8;                   // row stride in uint4
  float sum[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) sum[j] = 0.0f;
  float den;
  if (which && weights1 != nullptr) {
    float wsum = 0.0f;
#pragma unroll 4
    for (int i = 0; i < chunk; ++i) {
      const float w = weights1[base + i];
      const uint4 v = __ldg(x + i * rs);
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        sum[2 * j] = __fadd_rn(sum[2 * j], __fmul_rn(__uint_as_float(u[j] << 16), w));
        sum[2 * j + 1] = __fadd_rn(sum[2 * j + 1], __fmul_rn(__uint_as_float(u[j] & 0xffff0000u), w));
      }
      wsum = __fadd_rn(wsum, w);
    }
    den = wsum < 1.0f ? 1.0f : wsum;
  } else {
    const uint64_t* vbits = which ? bits1 : bits0;
    int cnt = 0;
#pragma unroll 4
    for (int i = 0; i < chunk; ++i) {
      const int64_t sidx = base + i;
      if (vbits != nullptr && !((vbits[sidx >> 6] >> (sidx & 63)) & 1ull)) continue;
      const uint4 v = __ldg(x + i * rs);
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        sum[2 * j] = __fadd_rn(sum[2 * j], __uint_as_float(u[j] << 16));
        sum[2 * j + 1] = __fadd_rn(sum[2 * j + 1], __uint_as_float(u[j] & 0xffff0000u));
      }
      ++cnt;
    }
    den = cnt > 0 ? (float)cnt : 1.0f;
  }
  float4* out = reinterpret_cast<float4*>((which ? out1 : out0) + ((int64_t)h * n + c) * D + dg);
  out[0] = make_float4(__fdiv_rn(sum[0], den), __fdiv_rn(sum[1], den), __fdiv_rn(sum[2], den),
                       __fdiv_rn(sum[3], den));
  out[1] = make_float4(__fdiv_rn(sum[4], den), __fdiv_rn(sum[5], den), __fdiv_rn(sum[6], den),
                       __fdiv_rn(sum[7], den));
}

// grid of pool_chunk_kernel for n chunks of D channels
static inline unsigned pool_blocks(int n, int D) {
  const int cpb = kPoolThreads / (D / 8);
  return (unsigned)((n + cpb - 1) / cpb);
}

// ================================================================ guided selection
// Score guidance of the uniform path: per key chunk c a scale 1 + boost_c that
// multiplies every score of column c before the selection
// (_attention_bsa.forward, bsa_interface.py:626-627; _attention_bsa_audio_guided
// .forward, :736-764).  Keys in chunk order; row r valid iff bit r of k_bits
// (nullptr = every row valid).

__device__ __forceinline__ bool row_valid(const uint64_t* bits, int64_t r) {
  return bits == nullptr || ((bits[r >> 6] >> (r & 63)) & 1ull);
}

// compute_channel_variance_density (bsa_interface.py:973-1062), one CTA per key
// chunk, thread d = channel d.  x_avg[r][d] = (sequential sum over heads) / heads;
// chunk channel means and frame means (ct frames of ch*cw rows) over the valid
// rows / max(count, 1); spatial = mean over d of (cm_d - mean_d cm)^2; temporal =
// mean over d of (sum over frame pairs with both frames non-empty of
// (fm[f+1] - fm[f])^2) / max(pairs, 1) (0 when ct == 1).  The means over d are
// sequential sums by thread 0, divided by D.  Writes spatial + temporal.
__global__ void variance_chunk_kernel(const uint16_t* __restrict__ v, int heads, int64_t Sk, int D,
                                      int chunk, int frame, const uint64_t* __restrict__ k_bits,
                                      float* __restrict__ combined) {
  __shared__ float red[2][256];
  __shared__ float gmean;
  const int c = blockIdx.x, d = threadIdx.x;
  const int64_t base = (int64_t)c * chunk;
  const float fh = (float)heads;
  float csum = 0.0f, fsum = 0.0f, prev = 0.0f, tsum = 0.0f;
  int ccnt = 0, fcnt = 0, pairs = 0;
  bool prev_ok = false;
  for (int i = 0; i < chunk; ++i) {
    const int64_t r = base + i;
    if (row_valid(k_bits, r)) {
      const uint16_t* p = v + r * D + d;
      float xs = 0.0f;
#pragma unroll 4
      for (int h = 0; h < heads; ++h) xs = __fadd_rn(xs, bfbits2f(p[(int64_t)h * Sk * D]));
      const float xa = __fdiv_rn(xs, fh);
      csum = __fadd_rn(csum, xa);
      fsum = __fadd_rn(fsum, xa);
      ++ccnt;
      ++fcnt;
    }
    if ((i + 1) % frame == 0) {  // frame end
      const float fm = __fdiv_rn(fsum, fcnt > 0 ? (float)fcnt : 1.0f);
      const bool ok = fcnt > 0;
      if (i + 1 > frame && ok && prev_ok) {
        const float df = __fsub_rn(fm, prev);
        tsum = __fadd_rn(tsum, __fmul_rn(df, df));
      }
      if (i + 1 > frame) pairs += (ok && prev_ok);
      prev = fm;
      prev_ok = ok;
      fsum = 0.0f;
      fcnt = 0;
    }
  }
  const float cm = __fdiv_rn(csum, ccnt > 0 ? (float)ccnt : 1.0f);
  const int n_frames = chunk / frame;
  const float tv = n_frames > 1 ? __fdiv_rn(tsum, pairs > 0 ? (float)pairs : 1.0f) : 0.0f;
  red[0][d] = cm;
  red[1][d] = tv;
  __syncthreads();
  if (d == 0) {
    float s = 0.0f;
    for (int j = 0; j < D; ++j) s = __fadd_rn(s, red[0][j]);
    gmean = __fdiv_rn(s, (float)D);
  }
  __syncthreads();
  const float dv = __fsub_rn(cm, gmean);
  __syncthreads();
  red[0][d] = __fmul_rn(dv, dv);
  __syncthreads();
  if (d == 0) {
    float s = 0.0f, t = 0.0f;
    for (int j = 0; j < D; ++j) s = __fadd_rn(s, red[0][j]);
    for (int j = 0; j < D; ++j) t = __fadd_rn(t, red[1][j]);
    const float spatial = __fdiv_rn(s, (float)D);
    const float temporal = n_frames > 1 ? __fdiv_rn(t, (float)D) : 0.0f;
    combined[c] = __fadd_rn(spatial, temporal);
  }
}

// x[c] /= max(max_c x[c], floor), one CTA (rho = combined / combined.max().clamp(min=1e-6),
// bsa_interface.py:1059-1060; block_means / max_val, :1100-1101).
__global__ void __launch_bounds__(1024) normalize_max_kernel(float* __restrict__ x, int64_t n,
                                                             float floor_) {
  __shared__ float red[32];
  float m = -INFINITY;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, x[i]);
  for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : -INFINITY;
    for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (threadIdx.x == 0) red[0] = m < floor_ ? floor_ : m;
  }
  __syncthreads();
  const float den = red[0];
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) x[i] = __fdiv_rn(x[i], den);
}

// compute_block_audio_saliency's block means (bsa_interface.py:1094-1098): sequential
// sum of the valid rows' norms / max(count, 1), one thread per chunk.
__global__ void chunk_mean_kernel(const float* __restrict__ x, int64_t n_chunks, int chunk,
                                  const uint64_t* __restrict__ k_bits, float* __restrict__ out) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= n_chunks) return;
  float s = 0.0f;
  int cnt = 0;
  for (int i = 0; i < chunk; ++i) {
    const int64_t r = c * chunk + i;
    if (!row_valid(k_bits, r)) continue;
    s = __fadd_rn(s, x[r]);
    ++cnt;
  }
  out[c] = __fdiv_rn(s, cnt > 0 ? (float)cnt : 1.0f);
}

// Path B weights (audio_weighted_mean_pooling_compression, bsa_interface.py:944-961):
// w = (1 + lambda * (a / max(1e-6, max of the chunk's valid a))) on valid rows, 0
// elsewhere; one thread per chunk.
__global__ void audio_pool_weights_kernel(const float* __restrict__ a, int64_t n_chunks, int chunk,
                                          const uint64_t* __restrict__ k_bits, float lambda_w,
                                          float* __restrict__ w) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= n_chunks) return;
  float mx = -1e9f;
  for (int i = 0; i < chunk; ++i) {
    const int64_t r = c * chunk + i;
    if (row_valid(k_bits, r)) mx = fmaxf(mx, a[r]);
  }
  if (mx < 1e-6f) mx = 1e-6f;
  for (int i = 0; i < chunk; ++i) {
    const int64_t r = c * chunk + i;
    w[r] = row_valid(k_bits, r) ? __fadd_rn(1.0f, __fmul_rn(lambda_w, __fdiv_rn(a[r], mx))) : 0.0f;
  }
}

// 1 + boost per key chunk, in the reference's order of operations:
//   ext   = modifier[c] (+ var_gamma * rho[c])  or  var_gamma * rho[c]   (:1467-1470)
//   boost = audio_gamma * (g * sal[c] + (1 - g) * uni)  (+ ext)           (:748-762)
//   scale = 1 + boost                                                     (:764, :1243-1245)
__global__ void guidance_scale_kernel(int64_t n, const float* __restrict__ rho, float var_gamma,
                                      const float* __restrict__ sal, const float* __restrict__ gate,
                                      float audio_gamma, float uni, const float* __restrict__ modifier,
                                      float* __restrict__ scale) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= n) return;
  bool has_ext = false;
  float ext = 0.0f;
  if (modifier != nullptr) {
    ext = modifier[c];
    has_ext = true;
  }
  if (rho != nullptr) {
    const float t = __fmul_rn(var_gamma, rho[c]);
    ext = has_ext ? __fadd_rn(ext, t) : t;
    has_ext = true;
  }
  float boost = 0.0f;
  if (sal != nullptr) {
    const float g = gate != nullptr ? *gate : 1.0f;
    const float gs = __fadd_rn(__fmul_rn(g, sal[c]), __fmul_rn(__fsub_rn(1.0f, g), uni));
    boost = __fmul_rn(audio_gamma, gs);
  }
  if (has_ext) boost = __fadd_rn(boost, ext);
  scale[c] = __fadd_rn(1.0f, boost);
}

// Per-token scalar gather into a chunk order (0 at padding), like gather_rows.
__global__ void gather_values_kernel(const float* __restrict__ x, int T, int H, int W, int Hp, int Wp,
                                     const int32_t* __restrict__ src_idx, int64_t n_rows,
                                     float* __restrict__ out) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n_rows) return;
  const int64_t g = src_idx[r];
  const int t = (int)(g / ((int64_t)Hp * Wp));
  const int hh = (int)((g / Wp) % Hp);
  const int w = (int)(g % Wp);
  out[r] = (t < T && hh < H && w < W) ? x[((int64_t)t * H + hh) * W + w] : 0.0f;
}

}  // namespace prism

using namespace prism;

// ===================================================================== C ABI
extern "C" {

const char* prism_last_error(void) { return prism::last_error(); }
int prism_abi_version(void) { return 5; }

prism_status_t prism_token_norms(const void* x, int64_t n_tokens, int dim, void* out,
                                 cudaStream_t stream) {
  PRISM_CHECK_ARG(x && out, "prism_token_norms: null pointer");
  PRISM_CHECK_ARG(n_tokens >= 0 && dim > 0 && dim % 8 == 0, "prism_token_norms: dim %d must be a positive multiple of 8", dim);
  PRISM_CHECK_ARG(aligned16(x), "prism_token_norms: x must be 16-byte aligned");
  if (n_tokens == 0) return PRISM_OK;
  const int threads = 256;
  const int64_t blocks = (n_tokens * 32 + threads - 1) / threads;
  token_norms_kernel<<<(unsigned)blocks, threads, 0, stream>>>(
      (const uint16_t*)x, n_tokens, dim, (__nv_bfloat16*)out);
  PRISM_CHECK_LAUNCH("prism_token_norms");
  return PRISM_OK;
}

size_t prism_zone_stats_workspace_bytes(int Tp, int Hp, int Wp, int D) {
  const size_t nz = (size_t)(Tp / 8) * (Hp / 8) * (Wp / 8);
  return nz * 8 * (size_t)kPart * ((size_t)D + 1) * sizeof(float);
}

prism_status_t prism_zone_stats(const void* v, int heads, int64_t v_stride_h, int64_t v_stride_s,
                                int T, int H, int W, int Tp, int Hp, int Wp, int D,
                                const uint8_t* valid, const void* norms, void* workspace,
                                float* packed, uint8_t* axis_valid, float* audio,
                                cudaStream_t stream) {
  PRISM_CHECK_ARG(v && workspace && packed && axis_valid && audio, "prism_zone_stats: null pointer");
  PRISM_CHECK_ARG(Tp > 0 && Hp > 0 && Wp > 0 && Tp % 8 == 0 && Hp % 8 == 0 && Wp % 8 == 0,
                  "prism_zone_stats: grid (%d,%d,%d) must be positive multiples of 8", Tp, Hp, Wp);
  PRISM_CHECK_ARG(heads >= 1 && D >= 2 && D % 2 == 0 && D <= 2048, "prism_zone_stats: bad heads/D");
  PRISM_CHECK_ARG(T >= 1 && H >= 1 && W >= 1 && T <= Tp && H <= Hp && W <= Wp && Tp - T < 8 &&
                  Hp - H < 8 && Wp - W < 8, "prism_zone_stats: source grid (%d,%d,%d) does not pad to (%d,%d,%d)",
                  T, H, W, Tp, Hp, Wp);
  PRISM_CHECK_ARG(v_stride_s % 2 == 0 && v_stride_h % 2 == 0 && ((uintptr_t)v & 3) == 0,
                  "prism_zone_stats: v must allow 4-byte channel-pair loads");
  const int Nz = (Tp / 8) * (Hp / 8) * (Wp / 8);
  float* part = (float*)workspace;
  float* apart = part + (size_t)Nz * 8 * kPart * D;
  if (D >= 16 && D <= 128) {  // 4 D >= 64 threads: one per token of the frame for the audio sums
    zone_partial_rows_kernel<<<Nz * 8, 4 * D, (size_t)72 * D * sizeof(float), stream>>>(
        (const uint16_t*)v, heads, v_stride_h, v_stride_s, T, H, W, Hp, Wp, D, valid,
        (const uint16_t*)norms, part, apart);
  } else {
    zone_partial_kernel<<<Nz * 8, D / 2, 0, stream>>>((const uint16_t*)v, heads, v_stride_h, v_stride_s,
                                                      T, H, W, Hp, Wp, D, valid, (const uint16_t*)norms,
                                                      part, apart);
  }
  PRISM_CHECK_LAUNCH("prism_zone_stats/partial");
  zone_combine_kernel<<<Nz, D < 1024 ? (D < 32 ? 32 : D) : 1024, 0, stream>>>(
      part, apart, T, H, W, Hp, Wp, D, valid, packed, axis_valid, audio);
  PRISM_CHECK_LAUNCH("prism_zone_stats/combine");
  return PRISM_OK;
}

prism_status_t prism_shape_select(const float* packed, const uint8_t* axis_valid,
                                  const float* audio, int has_audio, int Nz, int D, int method,
                                  float lambda_a, float tau_128, float lambda_128,
                                  int64_t* shape_ids, float* g_out, float* rho_out,
                                  cudaStream_t stream) {
  PRISM_CHECK_ARG(packed && axis_valid && shape_ids && (audio || !has_audio), "prism_shape_select: null pointer");
  PRISM_CHECK_ARG(method == 0 || method == 1, "prism_shape_select: unknown dynamic-block method %d", method);
  PRISM_CHECK_ARG(Nz >= 1 && Nz <= 6000, "prism_shape_select: Nz=%d outside [1, 6000]", Nz);
  // per-zone values (8 floats) + one row block of 6 x D channel terms per warp
  const size_t base = (size_t)Nz * 8 * sizeof(float), per_warp = (size_t)6 * D * sizeof(float);
  int warps = 16;
  while (warps > 1 && base + warps * per_warp > 227 * 1024) warps >>= 1;
  const size_t smem = base + warps * per_warp;
  PRISM_CHECK_ARG(smem <= 227 * 1024, "prism_shape_select: Nz=%d with D=%d exceeds shared memory", Nz, D);
  if (smem > 48 * 1024)
    PRISM_CHECK_CUDA(cudaFuncSetAttribute(shape_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                     "prism_shape_select: smem attribute");
  shape_select_kernel<<<1, warps * 32, smem, stream>>>(packed, axis_valid, audio, has_audio, Nz, D, method,
                                                 lambda_a, tau_128, lambda_128, shape_ids, g_out,
                                                 rho_out);
  PRISM_CHECK_LAUNCH("prism_shape_select");
  return PRISM_OK;
}

prism_status_t prism_build_layout(const int64_t* shape_ids, int Tp, int Hp, int Wp,
                                  int32_t* src_idx, int32_t* inv_idx, int32_t* block_of_tile,
                                  int32_t* block_tiles, int32_t* n_blocks, cudaStream_t stream) {
  PRISM_CHECK_ARG(shape_ids && src_idx && inv_idx && block_of_tile && block_tiles && n_blocks,
                  "prism_build_layout: null pointer");
  PRISM_CHECK_ARG(Tp > 0 && Hp > 0 && Wp > 0 && Tp % 8 == 0 && Hp % 8 == 0 && Wp % 8 == 0,
                  "prism_build_layout: grid (%d,%d,%d) must be positive multiples of 8", Tp, Hp, Wp);
  const int64_t S = (int64_t)Tp * Hp * Wp;
  PRISM_CHECK_ARG(S < (int64_t)1 << 31, "prism_build_layout: sequence too long for int32 indices");
  const int Nz = (int)(S / 512);
  block_map_kernel<<<1, 1024, 0, stream>>>(shape_ids, Nz, block_of_tile, block_tiles, n_blocks);
  PRISM_CHECK_LAUNCH("prism_build_layout/blocks");
  perm_kernel<<<(unsigned)((S + 255) / 256), 256, 0, stream>>>(shape_ids, Hp, Wp, S, src_idx, inv_idx);
  PRISM_CHECK_LAUNCH("prism_build_layout/perm");
  return PRISM_OK;
}

prism_status_t prism_tile_valid(const int32_t* src_idx, int64_t n_rows, const uint8_t* valid, int T,
                                int H, int W, int Tp, int Hp, int Wp, uint64_t* tile_bits,
                                int32_t* tile_count, cudaStream_t stream) {
  PRISM_CHECK_ARG(src_idx && tile_bits && tile_count, "prism_tile_valid: null pointer");
  PRISM_CHECK_ARG(Tp > 0 && Hp > 0 && Wp > 0 && T <= Tp && H <= Hp && W <= Wp,
                  "prism_tile_valid: bad grids");
  PRISM_CHECK_ARG(n_rows >= 0 && n_rows % 64 == 0, "prism_tile_valid: row count must be a multiple of 64");
  const int64_t nt = n_rows / 64;
  tile_valid_kernel<<<(unsigned)((nt * 32 + 255) / 256), 256, 0, stream>>>(src_idx, valid, nt, T, H, W, Hp, Wp,
                                                                            tile_bits, tile_count);
  PRISM_CHECK_LAUNCH("prism_tile_valid");
  return PRISM_OK;
}

prism_status_t prism_gather_rows(const void* x, int64_t x_stride_h, int64_t x_stride_s, int heads,
                                 int D, int T, int H, int W, int Tp, int Hp, int Wp,
                                 const int32_t* src_idx, int64_t n_rows, void* out,
                                 int64_t out_stride_h, cudaStream_t stream) {
  PRISM_CHECK_ARG(x && src_idx && out, "prism_gather_rows: null pointer");
  PRISM_CHECK_ARG(D % 8 == 0 && x_stride_h % 8 == 0 && x_stride_s % 8 == 0 && out_stride_h % 8 == 0 &&
                  aligned16(x) && aligned16(out), "prism_gather_rows: rows must be 16-byte aligned (D %% 8 == 0)");
  PRISM_CHECK_ARG(T >= 1 && H >= 1 && W >= 1 && T <= Tp && H <= Hp && W <= Wp,
                  "prism_gather_rows: bad grids");
  const int chunks = D / 8;
  PRISM_CHECK_ARG(n_rows >= 0 && n_rows * chunks < (int64_t)1 << 31 && heads <= 65535 &&
                      (int64_t)Tp * Hp * Wp < (int64_t)1 << 31,
                  "prism_gather_rows: bad row count");
  const int64_t total = n_rows * chunks;
  if (total == 0 || heads == 0) return PRISM_OK;
  if (x_stride_h == D && heads >= 2 && (int64_t)kTokRows * heads * chunks < (int64_t)1 << 31) {
    gather_rows_tok_kernel<<<(unsigned)((n_rows + kTokRows - 1) / kTokRows), 256, 0, stream>>>(
        (const uint4*)x, x_stride_s, heads, chunks, T, H, W, Hp, Wp, (int)n_rows, src_idx, (uint4*)out,
        out_stride_h);
  } else if (256 % chunks == 0) {
    const int64_t per_block = (256 / chunks) * kRowsPerThread;
    gather_rows4_kernel<<<dim3((unsigned)((n_rows + per_block - 1) / per_block), heads), 256, 0, stream>>>(
        (const uint4*)x, x_stride_h, x_stride_s, chunks, T, H, W, Hp, Wp, (int)n_rows, src_idx,
        (uint4*)out, out_stride_h);
  } else {
    gather_rows_kernel<<<dim3((unsigned)((total + 255) / 256), heads), 256, 0, stream>>>(
        (const uint4*)x, x_stride_h, x_stride_s, chunks, T, H, W, Hp, Wp, (int)n_rows, src_idx,
        (uint4*)out, out_stride_h);
  }
  PRISM_CHECK_LAUNCH("prism_gather_rows");
  return PRISM_OK;
}

prism_status_t prism_scatter_rows(const void* x_re, int64_t x_stride_h, int heads, int D, int T,
                                  int H, int W, int Tp, int Hp, int Wp, const int32_t* inv_idx,
                                  void* out, int64_t out_stride_h, int64_t out_stride_s,
                                  cudaStream_t stream) {
  PRISM_CHECK_ARG(x_re && inv_idx && out, "prism_scatter_rows: null pointer");
  PRISM_CHECK_ARG(D % 8 == 0 && x_stride_h % 8 == 0 && out_stride_h % 8 == 0 && out_stride_s % 8 == 0 &&
                  aligned16(x_re) && aligned16(out), "prism_scatter_rows: rows must be 16-byte aligned (D %% 8 == 0)");
  PRISM_CHECK_ARG(T <= Tp && H <= Hp && W <= Wp, "prism_scatter_rows: bad grids");
  const int64_t S = (int64_t)T * H * W;
  const int chunks = D / 8;
  PRISM_CHECK_ARG(S * chunks < (int64_t)1 << 31 && heads <= 65535, "prism_scatter_rows: too many rows");
  const int64_t total = S * chunks;
  if (total == 0 || heads == 0) return PRISM_OK;
  if (out_stride_h == D && heads >= 2 && (int64_t)kTokRows * heads * chunks < (int64_t)1 << 31) {
    scatter_rows_tok_kernel<<<(unsigned)((S + kTokRows - 1) / kTokRows), 256, 0, stream>>>(
        (const uint4*)x_re, x_stride_h, heads, chunks, T, H, W, Hp, Wp, inv_idx, (uint4*)out, out_stride_s);
  } else if (256 % chunks == 0) {
    const int64_t per_block = (256 / chunks) * kRowsPerThread;
    scatter_rows4_kernel<<<dim3((unsigned)((S + per_block - 1) / per_block), heads), 256, 0, stream>>>(
        (const uint4*)x_re, x_stride_h, chunks, T, H, W, Hp, Wp, inv_idx, (uint4*)out, out_stride_h,
        out_stride_s);
  } else {
    scatter_rows_kernel<<<dim3((unsigned)((total + 255) / 256), heads), 256, 0, stream>>>(
        (const uint4*)x_re, x_stride_h, chunks, T, H, W, Hp, Wp, inv_idx, (uint4*)out,
        out_stride_h, out_stride_s);
  }
  PRISM_CHECK_LAUNCH("prism_scatter_rows");
  return PRISM_OK;
}

prism_status_t prism_copy_rows(const void* src, int64_t src_stride_block, int64_t src_stride_row,
                               void* dst, int64_t dst_stride_block, int64_t dst_stride_row,
                               int64_t n_blocks, int64_t n_rows, int64_t row_bytes, cudaStream_t stream) {
  PRISM_CHECK_ARG(src && dst, "prism_copy_rows: null pointer");
  PRISM_CHECK_ARG(aligned16(src) && aligned16(dst) && row_bytes % 16 == 0 && src_stride_block % 16 == 0 &&
                      src_stride_row % 16 == 0 && dst_stride_block % 16 == 0 && dst_stride_row % 16 == 0,
                  "prism_copy_rows: pointers, strides and row length must be multiples of 16 bytes");
  PRISM_CHECK_ARG(n_blocks >= 0 && n_blocks <= 65535 && n_rows >= 0 && row_bytes >= 0 &&
                      row_bytes / 16 * kCopyRows < ((int64_t)1 << 31) &&
                      (n_rows + kCopyRows - 1) / kCopyRows < ((int64_t)1 << 31),
                  "prism_copy_rows: bad sizes");
  if (n_blocks == 0 || n_rows == 0 || row_bytes == 0) return PRISM_OK;
  copy_rows_kernel<<<dim3((unsigned)((n_rows + kCopyRows - 1) / kCopyRows), (unsigned)n_blocks), 256, 0,
                     stream>>>((const uint4*)src, src_stride_block / 16, src_stride_row / 16, (uint4*)dst,
                               dst_stride_block / 16, dst_stride_row / 16, n_rows, (int)(row_bytes / 16));
  PRISM_CHECK_LAUNCH("prism_copy_rows");
  return PRISM_OK;
}

size_t prism_block_select_workspace_bytes(int heads, int64_t S, int D) {
  const size_t nb_max = (size_t)(S / 64);
  size_t b = 2 * (size_t)heads * nb_max * D * sizeof(float);  // pooled q, k
  b += (size_t)heads * nb_max * nb_max * sizeof(float);       // scores
  b += (nb_max + 255) / 256 * 256;                            // block valid
  return b;
}

prism_status_t prism_block_select(const void* q_re, const void* k_re, int heads, int64_t S, int D,
                                  const int32_t* block_tiles, const int32_t* n_blocks,
                                  const uint64_t* tile_bits, int mode, double sparsity,
                                  double cdf_threshold, void* workspace, uint32_t* bits_q,
                                  uint32_t* bits_k, cudaStream_t stream) {
  PRISM_CHECK_ARG(q_re && k_re && block_tiles && n_blocks && tile_bits && workspace && bits_q && bits_k,
                  "prism_block_select: null pointer");
  PRISM_CHECK_ARG(mode >= 0 && mode <= 2, "prism_block_select: Either sparsity or cdf_threshold must be provided");
  PRISM_CHECK_ARG(S > 0 && S % 512 == 0, "prism_block_select: S must be a positive multiple of 512");
  PRISM_CHECK_ARG(D >= 16 && D <= 256, "prism_block_select: D=%d unsupported", D);
  const int64_t n_tiles = S / 64;
  const int nb_max = (int)n_tiles;
  PRISM_CHECK_ARG(nb_max <= 18000, "prism_block_select: %d blocks exceed the per-row shared-memory limit (18000)", nb_max);
  const int wq = (int)((n_tiles + 31) / 32);
  float* qc = (float*)workspace;
  float* kc = qc + (size_t)heads * nb_max * D;
  float* sc = kc + (size_t)heads * nb_max * D;
  uint8_t* bvalid = (uint8_t*)(sc + (size_t)heads * nb_max * nb_max);
  if (D % 2 == 0 && aligned_to(q_re, 4) && aligned_to(k_re, 4)) {
    pool2_kernel<<<dim3(nb_max, heads), D / 2, 0, stream>>>((const uint16_t*)q_re, (const uint16_t*)k_re, S,
                                                            D, block_tiles, n_blocks, tile_bits, qc, kc,
                                                            bvalid, nb_max);
  } else {
    pool_kernel<<<dim3(nb_max, heads), D, 0, stream>>>((const uint16_t*)q_re, (const uint16_t*)k_re, S, D,
                                                      block_tiles, n_blocks, tile_bits, qc, kc, bvalid,
                                                      nb_max);
  }
  PRISM_CHECK_LAUNCH("prism_block_select/pool");
  const size_t ssm = 2 * (size_t)D * (kScoreTile + 4) * sizeof(float);
  PRISM_CHECK_CUDA(cudaFuncSetAttribute(score_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ssm),
                   "prism_block_select: smem attribute");
  const int nt = (nb_max + kScoreTile - 1) / kScoreTile;
  score_kernel<<<dim3(nt, nt, heads), 256, ssm, stream>>>(qc, kc, D, n_blocks, nb_max, nb_max,
                                                          nullptr, sc);
  PRISM_CHECK_LAUNCH("prism_block_select/score");
  const float sm_scale = (float)(1.0 / sqrt((double)D));
  const size_t selsm = (size_t)nb_max * sizeof(unsigned long long) + ((size_t)nb_max + wq) * sizeof(uint32_t);
  PRISM_CHECK_CUDA(cudaFuncSetAttribute(select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)selsm),
                   "prism_block_select: smem attribute");
  select_kernel<<<dim3(nb_max, heads), kSelThreads, selsm, stream>>>(
      sc, bvalid, n_blocks, nb_max, nb_max, block_tiles, 2, 2, tile_bits, n_tiles, n_tiles, wq,
      mode, sparsity, cdf_threshold, sm_scale, bits_q);
  PRISM_CHECK_LAUNCH("prism_block_select/select");
  transpose_bits_kernel<<<dim3(wq, wq, heads), 32, 0, stream>>>(bits_q, n_tiles, n_tiles, wq, wq, bits_k);
  PRISM_CHECK_LAUNCH("prism_block_select/transpose");
  return PRISM_OK;
}

prism_status_t prism_uniform_layout(int Tp, int Hp, int Wp, int ct, int ch, int cw, int64_t n_rows,
                                    int32_t* src_idx, int32_t* inv_idx, cudaStream_t stream) {
  PRISM_CHECK_ARG(src_idx && inv_idx, "prism_uniform_layout: null pointer");
  PRISM_CHECK_ARG(ct > 0 && ch > 0 && cw > 0 && Tp > 0 && Hp > 0 && Wp > 0 && Tp % ct == 0 &&
                  Hp % ch == 0 && Wp % cw == 0,
                  "prism_uniform_layout: grid (%d,%d,%d) is not a multiple of the chunk (%d,%d,%d)",
                  Tp, Hp, Wp, ct, ch, cw);
  const int64_t Sp = (int64_t)Tp * Hp * Wp;
  PRISM_CHECK_ARG(n_rows >= Sp && n_rows < (int64_t)1 << 31,
                  "prism_uniform_layout: n_rows must cover the grid and stay below 2^31");
  uniform_perm_kernel<<<(unsigned)((n_rows + 255) / 256), 256, 0, stream>>>(Hp, Wp, ct, ch, cw, Sp,
                                                                             n_rows, src_idx, inv_idx);
  PRISM_CHECK_LAUNCH("prism_uniform_layout");
  return PRISM_OK;
}

size_t prism_block_select_uniform_workspace_bytes(int heads, int64_t n_chunks_q, int64_t n_chunks_k,
                                                  int D) {
  size_t b = (size_t)heads * (size_t)(n_chunks_q + n_chunks_k) * D * sizeof(float);  // pooled q, k
  b += (size_t)heads * (size_t)n_chunks_q * (size_t)n_chunks_k * sizeof(float);     // scores
  return b;
}

prism_status_t prism_block_select_uniform(const void* q_re, const void* k_re, int heads, int64_t Sq,
                                          int64_t Sk, int D, int64_t seq_q, int64_t seq_k,
                                          int chunk_q, int chunk_k, const uint64_t* q_bits,
                                          const uint64_t* k_bits, const float* k_weights,
                                          const float* col_scale, int mode, double sparsity,
                                          double cdf_threshold, void* workspace, uint32_t* bits_q,
                                          uint32_t* bits_k, cudaStream_t stream) {
  PRISM_CHECK_ARG(q_re && k_re && k_bits && workspace && bits_q && bits_k,
                  "prism_block_select_uniform: null pointer");
  PRISM_CHECK_ARG(mode >= 0 && mode <= 2, "prism_block_select_uniform: Either sparsity or cdf_threshold must be provided");
  PRISM_CHECK_ARG(Sq > 0 && Sq % 64 == 0 && Sk > 0 && Sk % 64 == 0 && heads >= 1,
                  "prism_block_select_uniform: sequence lengths must be positive multiples of 64");
  PRISM_CHECK_ARG(D >= 16 && D <= 256 && D % 8 == 0 && aligned16(q_re) && aligned16(k_re),
                  "prism_block_select_uniform: D=%d unsupported (16-byte rows, 16..256)", D);
  PRISM_CHECK_ARG(chunk_q > 0 && chunk_k > 0 && chunk_q % 64 == 0 && chunk_k % 64 == 0,
                  "prism_block_select_uniform: chunk sizes (%d, %d) must be multiples of 64 tokens",
                  chunk_q, chunk_k);
  PRISM_CHECK_ARG(seq_q > 0 && seq_q <= Sq && seq_q % chunk_q == 0 && seq_k > 0 && seq_k <= Sk &&
                      seq_k % chunk_k == 0,
                  "prism_block_select_uniform: sequences (%lld, %lld) are not whole numbers of chunks",
                  (long long)seq_q, (long long)seq_k);
  const int64_t n_qt = Sq / 64, n_kt = Sk / 64;
  const int nq = (int)(seq_q / chunk_q), nk = (int)(seq_k / chunk_k);
  PRISM_CHECK_ARG(nk <= 18000, "prism_block_select_uniform: %d key chunks exceed the per-row shared-memory limit (18000)", nk);
  const int wk = (int)((n_kt + 31) / 32), wq = (int)((n_qt + 31) / 32);
  float* qc = (float*)workspace;
  float* kc = qc + (size_t)heads * nq * D;
  float* sc = kc + (size_t)heads * nk * D;
  PRISM_CHECK_CUDA(cudaMemsetAsync(bits_q, 0, (size_t)heads * n_qt * wk * sizeof(uint32_t), stream),
                   "prism_block_select_uniform: clear bitmaps");
  pool_chunk_kernel<<<dim3(pool_blocks(nq > nk ? nq : nk, D), heads, 2), kPoolThreads, 0, stream>>>(
      (const uint16_t*)q_re, (const uint16_t*)k_re, Sq, Sk, D, chunk_q, nq, chunk_k, nk, q_bits,
      k_bits, k_weights, qc, kc);
  PRISM_CHECK_LAUNCH("prism_block_select_uniform/pool");
  const size_t ssm = 2 * (size_t)D * (kScoreTile + 4) * sizeof(float);
  PRISM_CHECK_CUDA(cudaFuncSetAttribute(score_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ssm),
                   "prism_block_select_uniform: smem attribute");
  score_kernel<<<dim3((nk + kScoreTile - 1) / kScoreTile, (nq + kScoreTile - 1) / kScoreTile, heads), 256,
                 ssm, stream>>>(qc, kc, D, nullptr, nq, nk, col_scale, sc);
  PRISM_CHECK_LAUNCH("prism_block_select_uniform/score");
  const float sm_scale = (float)(1.0 / sqrt((double)D));
  const size_t selsm = (size_t)nk * sizeof(unsigned long long) + ((size_t)nk + wk) * sizeof(uint32_t);
  PRISM_CHECK_CUDA(cudaFuncSetAttribute(select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)selsm),
                   "prism_block_select_uniform: smem attribute");
  select_kernel<<<dim3(nq, heads), kSelThreads, selsm, stream>>>(
      sc, nullptr, nullptr, nq, nk, nullptr, chunk_q / 64, chunk_k / 64, k_bits, n_qt, n_kt, wk, mode,
      sparsity, cdf_threshold, sm_scale, bits_q);
  PRISM_CHECK_LAUNCH("prism_block_select_uniform/select");
  transpose_bits_kernel<<<dim3(wq, wk, heads), 32, 0, stream>>>(bits_q, n_qt, n_kt, wq, wk, bits_k);
  PRISM_CHECK_LAUNCH("prism_block_select_uniform/transpose");
  return PRISM_OK;
}


// ------------------------------------------------------------ guided selection
prism_status_t prism_gather_values(const float* x, int T, int H, int W, int Tp, int Hp, int Wp,
                                   const int32_t* src_idx, int64_t n_rows, float* out,
                                   cudaStream_t stream) {
  PRISM_CHECK_ARG(x && src_idx && out, "prism_gather_values: null pointer");
  PRISM_CHECK_ARG(T >= 1 && H >= 1 && W >= 1 && T <= Tp && H <= Hp && W <= Wp,
                  "prism_gather_values: bad grids");
  PRISM_CHECK_ARG(n_rows >= 0 && n_rows < (int64_t)1 << 31, "prism_gather_values: bad row count");
  if (n_rows == 0) return PRISM_OK;
  gather_values_kernel<<<(unsigned)((n_rows + 255) / 256), 256, 0, stream>>>(x, T, H, W, Hp, Wp,
                                                                            src_idx, n_rows, out);
  PRISM_CHECK_LAUNCH("prism_gather_values");
  return PRISM_OK;
}

prism_status_t prism_variance_density(const void* v_re, int heads, int64_t Sk, int D, int64_t seq_k,
                                      int ct, int ch, int cw, const uint64_t* k_bits, float* rho,
                                      cudaStream_t stream) {
  PRISM_CHECK_ARG(v_re && rho, "prism_variance_density: null pointer");
  PRISM_CHECK_ARG(heads >= 1 && D >= 32 && D <= 256 && D % 32 == 0,
                  "prism_variance_density: D=%d must be a multiple of 32 in [32, 256]", D);
  PRISM_CHECK_ARG(ct >= 1 && ch >= 1 && cw >= 1, "prism_variance_density: bad chunk shape");
  const int chunk = ct * ch * cw;
  PRISM_CHECK_ARG(seq_k > 0 && seq_k <= Sk && seq_k % chunk == 0,
                  "prism_variance_density: %lld keys are not a whole number of %d-token chunks",
                  (long long)seq_k, chunk);
  const int64_t n = seq_k / chunk;
  PRISM_CHECK_ARG(n < (int64_t)1 << 31, "prism_variance_density: too many chunks");
  variance_chunk_kernel<<<(unsigned)n, D, 0, stream>>>((const uint16_t*)v_re, heads, Sk, D, chunk,
                                                       ch * cw, k_bits, rho);
  PRISM_CHECK_LAUNCH("prism_variance_density/chunks");
  normalize_max_kernel<<<1, 1024, 0, stream>>>(rho, n, 1e-6f);
  PRISM_CHECK_LAUNCH("prism_variance_density/normalize");
  return PRISM_OK;
}

prism_status_t prism_audio_saliency(const float* norms_re, int64_t seq_k, int chunk_k,
                                    const uint64_t* k_bits, float* saliency, cudaStream_t stream) {
  PRISM_CHECK_ARG(norms_re && saliency, "prism_audio_saliency: null pointer");
  PRISM_CHECK_ARG(chunk_k >= 1 && seq_k > 0 && seq_k % chunk_k == 0,
                  "prism_audio_saliency: %lld keys are not a whole number of %d-token chunks",
                  (long long)seq_k, chunk_k);
  const int64_t n = seq_k / chunk_k;
  chunk_mean_kernel<<<(unsigned)((n + 127) / 128), 128, 0, stream>>>(norms_re, n, chunk_k, k_bits,
                                                                     saliency);
  PRISM_CHECK_LAUNCH("prism_audio_saliency/means");
  normalize_max_kernel<<<1, 1024, 0, stream>>>(saliency, n, 1e-6f);
  PRISM_CHECK_LAUNCH("prism_audio_saliency/normalize");
  return PRISM_OK;
}

prism_status_t prism_audio_pool_weights(const float* norms_re, int64_t seq_k, int chunk_k,
                                        const uint64_t* k_bits, float lambda_w, float* weights,
                                        cudaStream_t stream) {
  PRISM_CHECK_ARG(norms_re && weights, "prism_audio_pool_weights: null pointer");
  PRISM_CHECK_ARG(chunk_k >= 1 && seq_k > 0 && seq_k % chunk_k == 0,
                  "prism_audio_pool_weights: %lld keys are not a whole number of %d-token chunks",
                  (long long)seq_k, chunk_k);
  const int64_t n = seq_k / chunk_k;
  audio_pool_weights_kernel<<<(unsigned)((n + 127) / 128), 128, 0, stream>>>(norms_re, n, chunk_k,
                                                                             k_bits, lambda_w, weights);
  PRISM_CHECK_LAUNCH("prism_audio_pool_weights");
  return PRISM_OK;
}

prism_status_t prism_chunk_scores(const float* qc, const float* kc, int heads, int nq, int nk, int D,
                                  float* scores, cudaStream_t stream) {
  PRISM_CHECK_ARG(qc && kc && scores, "prism_chunk_scores: null pointer");
  PRISM_CHECK_ARG(heads >= 1 && nq >= 1 && nk >= 1 && D >= 16 && D <= 256, "prism_chunk_scores: bad sizes");
  const size_t ssm = 2 * (size_t)D * (kScoreTile + 4) * sizeof(float);
  PRISM_CHECK_CUDA(cudaFuncSetAttribute(score_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ssm),
                   "prism_chunk_scores: smem attribute");
  score_kernel<<<dim3((nk + kScoreTile - 1) / kScoreTile, (nq + kScoreTile - 1) / kScoreTile, heads), 256,
                 ssm, stream>>>(qc, kc, D, nullptr, nq, nk, nullptr, scores);
  PRISM_CHECK_LAUNCH("prism_chunk_scores");
  return PRISM_OK;
}

prism_status_t prism_pool_chunks(const void* x_re, int heads, int64_t S, int D, int64_t seq,
                                int chunk, const uint64_t* bits, const float* weights, float* out,
                                cudaStream_t stream) {
  PRISM_CHECK_ARG(x_re && out, "prism_pool_chunks: null pointer");
  PRISM_CHECK_ARG(heads >= 1 && D >= 8 && D <= 1024 && D % 8 == 0 && aligned16(x_re) && aligned16(out),
                  "prism_pool_chunks: D must be a multiple of 8 (16-byte rows)");
  PRISM_CHECK_ARG(chunk >= 1 && seq > 0 && seq <= S && seq % chunk == 0,
                  "prism_pool_chunks: %lld rows are not a whole number of %d-row chunks",
                  (long long)seq, chunk);
  const int64_t n = seq / chunk;
  PRISM_CHECK_ARG(n < (int64_t)1 << 31, "prism_pool_chunks: too many chunks");
  // the second tensor slot of pool_chunk_kernel (the one with weights); the first is empty
  pool_chunk_kernel<<<dim3(pool_blocks((int)n, D), heads, 2), kPoolThreads, 0, stream>>>(
      (const uint16_t*)x_re, (const uint16_t*)x_re, S, S, D, chunk, 0, chunk, (int)n, nullptr, bits,
      weights, out, out);
  PRISM_CHECK_LAUNCH("prism_pool_chunks");
  return PRISM_OK;
}

prism_status_t prism_guidance_scale(int64_t n_chunks, const float* rho, float variance_gamma,
                                    const float* saliency, const float* audio_gate, float audio_gamma,
                                    const float* modifier, float* scale, cudaStream_t stream) {
  PRISM_CHECK_ARG(scale && n_chunks > 0, "prism_guidance_scale: null pointer or no chunks");
  const float uni = (float)(1.0 / (double)n_chunks);
  guidance_scale_kernel<<<(unsigned)((n_chunks + 255) / 256), 256, 0, stream>>>(
      n_chunks, rho, variance_gamma, saliency, audio_gate, audio_gamma, uni, modifier, scale);
  PRISM_CHECK_LAUNCH("prism_guidance_scale");
  return PRISM_OK;
}

}  // extern "C"
