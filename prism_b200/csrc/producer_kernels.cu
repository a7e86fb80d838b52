// Producer side of the video self-attention (SelfAttention.forward,
// hymm/models/modules/wan_video_dit.py:699-705, 764-787): after the q / k / v
// projections, RMSNorm of q and k over the full hidden width (torch.nn.RMSNorm,
// :226-227), 3D RoPE of q and k in float64 complex arithmetic (rope_apply_head_dim,
// :177-182) and the Ulysses all-to-all pack (all_to_all_4D's send layout
// [P, S/P, H/P, D], head padding to P * hp heads, :775-787), fused into one pass
// per token row; and its backward.
//
// Numerics follow the reference's op sequence: the norm in fp32
// (x * rsqrt(mean(x^2) + eps)) * gamma rounded to bf16; the rotation of that bf16
// pair in double, (a c - b s, a s + b c); the double result rounded to float, then
// to bf16 (the double -> bf16 conversion goes through float).  Backward: the
// conjugate rotation in double rounded the same way, then the RMSNorm gradient in
// fp32.  Built with -fmad=false (every product and sum rounds once).
#include <cuda_bf16.h>
#include <math.h>
#include <stdint.h>

#include "prism_bsa.h"
#include "prism_common.cuh"

namespace prism {

constexpr int kProdThreads = 128;

__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(lo)) |
         ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(hi)) << 16);
}
// double -> bf16 as torch converts it: through float
__device__ __forceinline__ float d2bf(double x) {
  return __bfloat162float(__float2bfloat16_rn(__double2float_rn(x)));
}

__device__ float block_sum_f(float v, float* red) {
  for (int o = 16; o >= 1; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.0f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s = __fadd_rn(s, red[i]);
  return s;
}

// One CTA per packed row s < S_pack.  x rows [S, C] (C = H * D, row stride ld
// elements); out [P][S_pack][hp][D] with P * hp >= H (heads h >= H are zero, rows
// s >= S are zero: the last rank's padding of an uneven split).  norm = 0: v
// (copy); norm = 1: RMSNorm + RoPE.  rope_cs [S][D/2][2] doubles (cos, sin).
__global__ void __launch_bounds__(kProdThreads) norm_rope_pack_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t ld, int64_t S, int64_t S_pack, int H, int D, int P,
    int hp, const float* __restrict__ gamma, float eps, const double* __restrict__ rope_cs, int norm,
    __nv_bfloat16* __restrict__ out, float* __restrict__ rstd_out) {
  extern __shared__ double cs[];  // D/2 (cos, sin) pairs of this token
  __shared__ float red[32];
  const int64_t s = blockIdx.x;
  if (s >= S) {  // padding row (uniform per CTA)
    for (int i = threadIdx.x; i < P * hp * D / 8; i += blockDim.x) {
      const int col = i * 8, h = col / D, d0 = col - h * D, p = h / hp, hh = h - p * hp;
      reinterpret_cast<uint4*>(out + (((int64_t)p * S_pack + s) * hp + hh) * D + d0)[0] = make_uint4(0, 0, 0, 0);
    }
    return;
  }
  const int C = H * D;
  const uint4* xr = reinterpret_cast<const uint4*>(x + s * ld);
  const int nv = C / 8;
  float r = 1.0f;
  if (norm) {
    for (int i = threadIdx.x; i < D; i += blockDim.x) cs[i] = rope_cs[s * D + i];
    float ss = 0.0f;
    for (int i = threadIdx.x; i < nv; i += blockDim.x) {
      const uint4 v = __ldg(xr + i);
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float a = bf_lo(u[j]), b = bf_hi(u[j]);
        ss = __fadd_rn(ss, __fadd_rn(__fmul_rn(a, a), __fmul_rn(b, b)));
      }
    }
    const float tot = block_sum_f(ss, red);
    r = rsqrtf(__fadd_rn(__fdiv_rn(tot, (float)C), eps));
    if (threadIdx.x == 0) rstd_out[s] = r;
    __syncthreads();  // cs visible
  }
  const int nvp = P * hp * D / 8;  // padded row of the packed layout
  for (int i = threadIdx.x; i < nvp; i += blockDim.x) {
    const int col = i * 8;
    const int h = col / D, d0 = col - h * D;
    uint4 o = make_uint4(0, 0, 0, 0);
    if (h < H) {
      const uint4 v = __ldg(xr + i);
      if (!norm) {
        o = v;
      } else {
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
        uint32_t w[4];
        const float4 g0 = gamma ? reinterpret_cast<const float4*>(gamma + col)[0] : make_float4(1, 1, 1, 1);
        const float4 g1 = gamma ? reinterpret_cast<const float4*>(gamma + col)[1] : make_float4(1, 1, 1, 1);
        const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          // normed pair, rounded to bf16 (the RMSNorm output dtype)
          const double a = (double)__bfloat162float(__float2bfloat16_rn(__fmul_rn(__fmul_rn(bf_lo(u[j]), r), g[2 * j])));
          const double b = (double)__bfloat162float(__float2bfloat16_rn(__fmul_rn(__fmul_rn(bf_hi(u[j]), r), g[2 * j + 1])));
          const int pi = (d0 >> 1) + j;
          const double c = cs[2 * pi], sn = cs[2 * pi + 1];
          const double re = __dsub_rn(__dmul_rn(a, c), __dmul_rn(b, sn));
          const double im = __dadd_rn(__dmul_rn(a, sn), __dmul_rn(b, c));
          w[j] = pack2(d2bf(re), d2bf(im));
        }
        o = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    const int p = h / hp, hh = h - p * hp;
    reinterpret_cast<uint4*>(out + (((int64_t)p * S_pack + s) * hp + hh) * D + d0)[0] = o;
  }
}

// Backward, kProdRows token rows per CTA.  g [P][S][hp][D]: gradient of the
// packed output.  norm = 0: dx = unpacked g.  norm = 1: dy = conj-rotated g
// (double, rounded to bf16 through float), then the RMSNorm gradient with
// r = rstd[s]: dx = r (gamma dy) - x r^3 / C * sum(gamma dy x); dgamma partials
// [gridDim.x][C] = sum over the CTA's rows of dy x r.
constexpr int kProdRows = 64;
template <int kMaxV>  // 8-column groups per thread: ceil(C / 8 / kProdThreads)
__global__ void __launch_bounds__(kProdThreads) norm_rope_pack_bwd_kernel(
    const __nv_bfloat16* __restrict__ g, const __nv_bfloat16* __restrict__ x, int64_t ld, int64_t S,
    int64_t S_pack, int H, int D, int P, int hp, const float* __restrict__ gamma, const float* __restrict__ rstd,
    const double* __restrict__ rope_cs, int norm, __nv_bfloat16* __restrict__ dx, int64_t ldx,
    float* __restrict__ dgamma_part) {
  extern __shared__ double cs[];
  __shared__ float red[32];
  const int C = H * D;
  const int nv = C / 8;
  // each thread owns the 8-column groups i = threadIdx.x + k * kProdThreads, k < kMaxV
  float dg[kMaxV][8];
#pragma unroll
  for (int k = 0; k < kMaxV; ++k)
#pragma unroll
    for (int j = 0; j < 8; ++j) dg[k][j] = 0.0f;
  const int64_t s0 = (int64_t)blockIdx.x * kProdRows;
  for (int rr = 0; rr < kProdRows; ++rr) {
    const int64_t s = s0 + rr;
    if (s >= S) break;
    if (!norm) {
      for (int i = threadIdx.x; i < nv; i += blockDim.x) {
        const int col = i * 8, h = col / D, d0 = col - h * D, p = h / hp, hh = h - p * hp;
        reinterpret_cast<uint4*>(dx + s * ldx + col)[0] =
            reinterpret_cast<const uint4*>(g + (((int64_t)p * S_pack + s) * hp + hh) * D + d0)[0];
      }
      continue;
    }
    __syncthreads();  // previous row's cs reads done
    for (int i = threadIdx.x; i < D; i += blockDim.x) cs[i] = rope_cs[s * D + i];
    __syncthreads();
    const float r = rstd[s];
    float dyv[kMaxV][8], xv[kMaxV][8];
    float dot = 0.0f;
#pragma unroll
    for (int k = 0; k < kMaxV; ++k) {
      const int i = threadIdx.x + k * kProdThreads;
      if (i >= nv) break;
      const int col = i * 8, h = col / D, d0 = col - h * D, p = h / hp, hh = h - p * hp;
      const uint4 gv = reinterpret_cast<const uint4*>(g + (((int64_t)p * S_pack + s) * hp + hh) * D + d0)[0];
      const uint4 xq = __ldg(reinterpret_cast<const uint4*>(x + s * ld) + i);
      const uint32_t gu[4] = {gv.x, gv.y, gv.z, gv.w};
      const uint32_t xu[4] = {xq.x, xq.y, xq.z, xq.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int pi = (d0 >> 1) + j;
        const double c = cs[2 * pi], sn = cs[2 * pi + 1];
        const double ga = (double)bf_lo(gu[j]), gb = (double)bf_hi(gu[j]);
        // gradient through (a + ib)(c + is): conj rotation
        dyv[k][2 * j] = d2bf(__dadd_rn(__dmul_rn(ga, c), __dmul_rn(gb, sn)));
        dyv[k][2 * j + 1] = d2bf(__dsub_rn(__dmul_rn(gb, c), __dmul_rn(ga, sn)));
        xv[k][2 * j] = bf_lo(xu[j]);
        xv[k][2 * j + 1] = bf_hi(xu[j]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float gm = gamma ? gamma[col + j] : 1.0f;
        dot = __fadd_rn(dot, __fmul_rn(__fmul_rn(gm, dyv[k][j]), xv[k][j]));
      }
    }
    const float tot = block_sum_f(dot, red);
    const float coef = __fdiv_rn(__fmul_rn(__fmul_rn(__fmul_rn(r, r), r), tot), (float)C);
#pragma unroll
    for (int k = 0; k < kMaxV; ++k) {
      const int i = threadIdx.x + k * kProdThreads;
      if (i >= nv) break;
      const int col = i * 8;
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float o[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int jj = 2 * j + e;
          const float gm = gamma ? gamma[col + jj] : 1.0f;
          o[e] = __fsub_rn(__fmul_rn(r, __fmul_rn(gm, dyv[k][jj])), __fmul_rn(xv[k][jj], coef));
          dg[k][jj] = __fadd_rn(dg[k][jj], __fmul_rn(dyv[k][jj], __fmul_rn(xv[k][jj], r)));
        }
        w[j] = pack2(o[0], o[1]);
      }
      reinterpret_cast<uint4*>(dx + s * ldx + col)[0] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  if (norm && dgamma_part != nullptr) {
#pragma unroll
    for (int k = 0; k < kMaxV; ++k) {
      const int i = threadIdx.x + k * kProdThreads;
      if (i >= nv) break;
      float4* dst = reinterpret_cast<float4*>(dgamma_part + (int64_t)blockIdx.x * C + i * 8);
      dst[0] = make_float4(dg[k][0], dg[k][1], dg[k][2], dg[k][3]);
      dst[1] = make_float4(dg[k][4], dg[k][5], dg[k][6], dg[k][7]);
    }
  }
}

// out[c] = sum over rows b of part[b][c] (sequential in b), one thread per column.
__global__ void column_sum_kernel(const float* __restrict__ part, int64_t rows, int C,
                                  float* __restrict__ out) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  float s = 0.0f;
#pragma unroll 8
  for (int64_t b = 0; b < rows; ++b) s = __fadd_rn(s, __ldg(part + b * C + c));
  out[c] = s;
}

}  // namespace prism

using namespace prism;

extern "C" {

prism_status_t prism_norm_rope_pack(const void* x, int64_t ld, int64_t S, int64_t S_pack, int H, int D,
                                    int P, int hp, const float* gamma, float eps, const double* rope_cs,
                                    int norm, void* out, float* rstd, cudaStream_t stream) {
  PRISM_CHECK_ARG(x && out && (!norm || (rope_cs && rstd)), "prism_norm_rope_pack: null pointer");
  PRISM_CHECK_ARG(S >= 0 && S_pack >= S && S_pack < (int64_t)1 << 31 && H >= 1 && D >= 8 && D % 8 == 0 &&
                      P >= 1 && hp >= 1 && P * hp >= H && ld % 8 == 0 && ld >= (int64_t)H * D,
                  "prism_norm_rope_pack: bad sizes");
  PRISM_CHECK_ARG(aligned16(x) && aligned16(out) && (gamma == nullptr || aligned16(gamma)),
                  "prism_norm_rope_pack: tensors must be 16-byte aligned");
  if (S_pack == 0) return PRISM_OK;
  norm_rope_pack_kernel<<<(unsigned)S_pack, kProdThreads, norm ? D * sizeof(double) : 0, stream>>>(
      (const __nv_bfloat16*)x, ld, S, S_pack, H, D, P, hp, gamma, eps, rope_cs, norm, (__nv_bfloat16*)out,
      rstd);
  PRISM_CHECK_LAUNCH("prism_norm_rope_pack");
  return PRISM_OK;
}

size_t prism_norm_rope_pack_bwd_workspace_bytes(int64_t S, int H, int D) {
  return (size_t)((S + kProdRows - 1) / kProdRows) * (size_t)H * D * sizeof(float);
}

prism_status_t prism_norm_rope_pack_bwd(const void* g, const void* x, int64_t ld, int64_t S, int64_t S_pack,
                                        int H, int D, int P, int hp, const float* gamma, const float* rstd,
                                        const double* rope_cs, int norm, void* dx, int64_t ldx,
                                        void* workspace, float* dgamma, cudaStream_t stream) {
  PRISM_CHECK_ARG(g && dx && (!norm || (x && rstd && rope_cs && workspace && dgamma)),
                  "prism_norm_rope_pack_bwd: null pointer");
  PRISM_CHECK_ARG(S >= 0 && S_pack >= S && H >= 1 && D >= 8 && D % 8 == 0 && P >= 1 && hp >= 1 && P * hp >= H &&
                      (int64_t)H * D <= 8 * 8 * kProdThreads && ld % 8 == 0 && ldx % 8 == 0,
                  "prism_norm_rope_pack_bwd: bad sizes (hidden width <= %d)", 8 * 8 * kProdThreads);
  PRISM_CHECK_ARG(aligned16(g) && aligned16(dx) && (x == nullptr || aligned16(x)) &&
                      (gamma == nullptr || aligned16(gamma)),
                  "prism_norm_rope_pack_bwd: tensors must be 16-byte aligned");
  if (S == 0) return PRISM_OK;
  const int64_t blocks = (S + kProdRows - 1) / kProdRows;
  const int nvt = (H * D / 8 + kProdThreads - 1) / kProdThreads;
  const size_t sm = norm ? D * sizeof(double) : 0;
  float* part = norm ? (float*)workspace : nullptr;
#define PRISM_NRP_BWD(V)                                                                              \
  norm_rope_pack_bwd_kernel<V><<<(unsigned)blocks, kProdThreads, sm, stream>>>(                        \
      (const __nv_bfloat16*)g, (const __nv_bfloat16*)x, ld, S, S_pack, H, D, P, hp, gamma, rstd, rope_cs,   \
      norm, (__nv_bfloat16*)dx, ldx, part)
  switch (nvt) {
    case 1: PRISM_NRP_BWD(1); break;
    case 2: PRISM_NRP_BWD(2); break;
    case 3: PRISM_NRP_BWD(3); break;
    case 4: PRISM_NRP_BWD(4); break;
    case 5: PRISM_NRP_BWD(5); break;
    case 6: PRISM_NRP_BWD(6); break;
    case 7: PRISM_NRP_BWD(7); break;
    default: PRISM_NRP_BWD(8); break;
  }
#undef PRISM_NRP_BWD
  PRISM_CHECK_LAUNCH("prism_norm_rope_pack_bwd");
  if (norm) {
    const int C = H * D;
    column_sum_kernel<<<(C + 255) / 256, 256, 0, stream>>>((const float*)workspace, blocks, C, dgamma);
    PRISM_CHECK_LAUNCH("prism_norm_rope_pack_bwd/dgamma");
  }
  return PRISM_OK;
}

}  // extern "C"
