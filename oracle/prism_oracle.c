/*
 * prism_oracle.c -- CPU restatement of Prism's dynamic block-shape block-sparse
 * attention path (selection side).  TEST INFRASTRUCTURE ONLY: this file is the
 * checker that the CUDA kernels in prism_b200/csrc are compared against.  The
 * product never links, loads or calls it.
 *
 * Every function follows one step of the reference and cites it
 * (paths are relative to the reference project root):
 *
 *   oracle_token_norms   hymm/models/modules/wan_video_dit.py:742-744
 *   oracle_zone_stats    block_sparse_attention/dynamic_block_attention.py:236,
 *                        block_sparse_attention/dynamic_block_shape.py:68-129,
 *                        dynamic_block_shape.py:189-245 (audio part)
 *   oracle_shape_select  dynamic_block_shape.py:248-391
 *   oracle_layout        dynamic_block_attention.py:21-63, 107-170
 *   oracle_block_select  bsa_interface.py:177-201, 203-207, 235-304,
 *                        dynamic_block_attention.py:173-188, 256-319
 *   oracle_block_select_uniform
 *                        bsa_interface.py:164-201, 203-207, 235-304, 600-633
 *                        (uniform fixed-shape path, flash_attn_bsa_3d :1123-1176;
 *                        guided: k pooling weights :902-970, score scale :626-627,
 *                        :736-764)
 *   oracle_variance_density   bsa_interface.py:973-1062
 *   oracle_audio_saliency     bsa_interface.py:1065-1102
 *   oracle_audio_pool_weights bsa_interface.py:902-970 (the weights)
 *   oracle_guidance_scale     bsa_interface.py:744-764, 1240-1245, 1467-1470
 *   oracle_uniform_pooled     bsa_interface.py:164-207 (pooled chunks, raw scores)
 *   oracle_correction_stats   bias_rectification.py:146-170, 421-436 (A_pool, R_n,
 *                             variance M, unselected chunks)
 *
 * Floating-point order.  The reference leaves summation order to torch; this
 * restatement fixes one order (the one the CUDA kernels use) so that GPU and
 * CPU agree bit for bit.  Build with -ffp-contract=off: every a*b+c below is
 * two roundings unless fmaf() is written out.
 *
 * Parity against the reference itself is pinned by tests/golden (fixtures
 * produced by running the reference's own Python code on CPU).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ bf16 */
static float bf16_to_f32(uint16_t b) {
  uint32_t u = ((uint32_t)b) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static uint16_t f32_to_bf16_rn(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* NaN */
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}

/* ------------------------------------------------- deterministic math
 * exp and log2 evaluated in double with only + - * / (each correctly rounded)
 * and exact scalings, then rounded once to float.  Same algorithm as the
 * device code; results are bit-identical on CPU and GPU.
 *
 * exp:  Cody-Waite argument reduction x = k*ln2 + r, |r| <= ln2/2, then the
 *       Taylor series of e^r to degree 13 (Horner), then scaling by 2^k.
 * log2: x = 2^e * m with m in [sqrt(1/2), sqrt(2)), ln m = 2*atanh(z),
 *       z = (m-1)/(m+1), atanh series to z^23, then log2 x = e + ln m / ln 2.
 */
static double pow2_int(int k) { /* 2^k for -1022 <= k <= 1023 */
  uint64_t bits = (uint64_t)(k + 1023) << 52;
  double d;
  memcpy(&d, &bits, 8);
  return d;
}

float oracle_det_expf(float xf) {
  if (xf == -INFINITY) return 0.0f;
  if (xf < -120.0f) return 0.0f;
  if (xf > 88.0f) return INFINITY;
  const double LN2_HI = 6.93147180369123816490e-01; /* ln2 split: hi has 32 bits */
  const double LN2_LO = 1.90821492927058770002e-10;
  const double INV_LN2 = 1.44269504088896338700e+00;
  double x = (double)xf;
  double kd = nearbyint(x * INV_LN2);
  int k = (int)kd;
  double r = (x - kd * LN2_HI) - kd * LN2_LO;
  /* Taylor: sum_{n=0}^{13} r^n / n!  (Horner) */
  double p = 1.0 / 6227020800.0; /* 1/13! */
  p = p * r + 1.0 / 479001600.0;
  p = p * r + 1.0 / 39916800.0;
  p = p * r + 1.0 / 3628800.0;
  p = p * r + 1.0 / 362880.0;
  p = p * r + 1.0 / 40320.0;
  p = p * r + 1.0 / 5040.0;
  p = p * r + 1.0 / 720.0;
  p = p * r + 1.0 / 120.0;
  p = p * r + 1.0 / 24.0;
  p = p * r + 1.0 / 6.0;
  p = p * r + 0.5;
  p = p * r + 1.0;
  p = p * r + 1.0;
  return (float)(p * pow2_int(k));
}

float oracle_det_log2f(float xf) {
  /* xf > 0 and normal (callers clamp to >= 1e-4) */
  uint32_t u;
  memcpy(&u, &xf, 4);
  int e = (int)((u >> 23) & 0xff) - 127;
  uint32_t mb = (u & 0x007fffffu) | 0x3f800000u;
  float mf;
  memcpy(&mf, &mb, 4);
  double m = (double)mf;
  if (m > 1.4142135623730951) { m = m * 0.5; e += 1; }
  double z = (m - 1.0) / (m + 1.0);
  double z2 = z * z;
  double s = 1.0 / 23.0;
  s = s * z2 + 1.0 / 21.0;
  s = s * z2 + 1.0 / 19.0;
  s = s * z2 + 1.0 / 17.0;
  s = s * z2 + 1.0 / 15.0;
  s = s * z2 + 1.0 / 13.0;
  s = s * z2 + 1.0 / 11.0;
  s = s * z2 + 1.0 / 9.0;
  s = s * z2 + 1.0 / 7.0;
  s = s * z2 + 1.0 / 5.0;
  s = s * z2 + 1.0 / 3.0;
  s = s * z2 + 1.0;
  double lnm = 2.0 * z * s;
  const double INV_LN2 = 1.44269504088896338700e+00;
  return (float)((double)e + lnm * INV_LN2);
}

/* -------------------------------------------------------- token norms
 * ||x[n]||_2 over `dim` channels, bf16 in / bf16 out.
 * Order (one 32-lane warp per token): lane l owns 8-element chunks
 * c = l, l+32, ...; within a chunk acc = fmaf(x, x, acc) sequentially;
 * then a butterfly over lanes (xor 16, 8, 4, 2, 1) of plain adds.
 * Reference: wan_video_dit.py:742-744 (a2v_bridge_residual.norm(dim=-1)).
 */
void oracle_token_norms(const uint16_t* x, int64_t n, int dim, uint16_t* out) {
  for (int64_t t = 0; t < n; ++t) {
    const uint16_t* row = x + t * (int64_t)dim;
    float acc[32];
    for (int l = 0; l < 32; ++l) {
      float a = 0.0f;
      for (int c = l; c * 8 < dim; c += 32)
        for (int j = 0; j < 8; ++j) {
          float v = bf16_to_f32(row[c * 8 + j]);
          a = fmaf(v, v, a);
        }
      acc[l] = a;
    }
    for (int off = 16; off >= 1; off >>= 1) {
      float nxt[32];
      for (int l = 0; l < 32; ++l) nxt[l] = acc[l] + acc[l ^ off];
      memcpy(acc, nxt, sizeof(acc));
    }
    out[t] = f32_to_bf16_rn(sqrtf(acc[0]));
  }
}

/* ---------------------------------------------------------- zone stats
 * v [heads, S, D] bf16 (THW order, padded), valid [S] (NULL = all valid),
 * norms [S] bf16 (NULL = no audio).
 * Outputs:
 *   packed      [Nz, 25*D] f32 : channel mean | T means [8,D] | H [8,D] | W [8,D]
 *   axis_valid  [Nz, 24] u8    : t_valid[8] | h_valid[8] | w_valid[8]
 *   audio       [Nz, 25]  f32  : a_bar | aT[8] | aH[8] | aW[8]  (masked means)
 * Head average: vavg = bf16( (sum_h v_h, sequential) / heads )
 *   (dynamic_block_attention.py:236 -- torch bf16 mean = fp32 sum / n, rounded).
 * Per (zone, local frame lt), per channel: rowH[lh] = sum_lw x (sequential lw),
 * frame = sum_lh rowH[lh], colW[lw] = sum_lh x (sequential lh); then the
 * zone sums combine the eight frames in order lt = 0..7.
 * Masked means as dynamic_block_shape.py:96-111 (count clamped to >= 1).
 */
void oracle_zone_stats(const uint16_t* v, int heads, int T, int H, int W, int D,
                       const uint8_t* valid, const uint16_t* norms,
                       float* packed, uint8_t* axis_valid, float* audio) {
  const int ZT = T / 8, ZH = H / 8, ZW = W / 8;
  const int Nz = ZT * ZH * ZW;
  const int64_t S = (int64_t)T * H * W;
  const int PK = 25 * D;
  float* rowH = (float*)malloc(sizeof(float) * 8 * 8 * D); /* [lt][lh][D] */
  float* colW = (float*)malloc(sizeof(float) * 8 * 8 * D); /* [lt][lw][D] */
  float* frame = (float*)malloc(sizeof(float) * 8 * D);    /* [lt][D] */
  for (int z = 0; z < Nz; ++z) {
    const int zt = z / (ZH * ZW), zh = (z / ZW) % ZH, zw = z % ZW;
    int cT[8] = {0}, cH[8] = {0}, cW[8] = {0}, call = 0;
    float arow[8][8], acol[8][8], aframe[8];
    for (int lt = 0; lt < 8; ++lt) {
      for (int d = 0; d < D; ++d) {
        float cw[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        float fr = 0.0f;
        for (int lh = 0; lh < 8; ++lh) {
          float rh = 0.0f;
          for (int lw = 0; lw < 8; ++lw) {
            int64_t s = ((int64_t)(zt * 8 + lt) * H + (zh * 8 + lh)) * W + (zw * 8 + lw);
            if (valid && !valid[s]) continue;
            float acc = 0.0f;
            for (int h = 0; h < heads; ++h) acc += bf16_to_f32(v[((int64_t)h * S + s) * D + d]);
            float x = bf16_to_f32(f32_to_bf16_rn(acc / (float)heads));
            rh += x;
            cw[lw] += x;
          }
          rowH[(lt * 8 + lh) * D + d] = rh;
          fr += rh;
        }
        for (int lw = 0; lw < 8; ++lw) colW[(lt * 8 + lw) * D + d] = cw[lw];
        frame[lt * D + d] = fr;
      }
      /* audio: one scalar per token, same structure */
      {
        float cw[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        float fr = 0.0f;
        for (int lh = 0; lh < 8; ++lh) {
          float rh = 0.0f;
          for (int lw = 0; lw < 8; ++lw) {
            int64_t s = ((int64_t)(zt * 8 + lt) * H + (zh * 8 + lh)) * W + (zw * 8 + lw);
            if (valid && !valid[s]) continue;
            cT[lt]++; cH[lh]++; cW[lw]++; call++;
            float x = norms ? bf16_to_f32(norms[s]) : 0.0f;
            rh += x;
            cw[lw] += x;
          }
          arow[lt][lh] = rh;
          fr += rh;
        }
        for (int lw = 0; lw < 8; ++lw) acol[lt][lw] = cw[lw];
        aframe[lt] = fr;
      }
    }
    float* pk = packed + (int64_t)z * PK;
    const float fall = (float)(call > 0 ? call : 1);
    for (int d = 0; d < D; ++d) {
      float cs = 0.0f;
      for (int lt = 0; lt < 8; ++lt) cs += frame[lt * D + d];
      pk[d] = cs / fall;
      for (int lt = 0; lt < 8; ++lt)
        pk[D + lt * D + d] = frame[lt * D + d] / (float)(cT[lt] > 0 ? cT[lt] : 1);
      for (int p = 0; p < 8; ++p) {
        float sh = 0.0f, sw = 0.0f;
        for (int lt = 0; lt < 8; ++lt) {
          sh += rowH[(lt * 8 + p) * D + d];
          sw += colW[(lt * 8 + p) * D + d];
        }
        pk[D + 8 * D + p * D + d] = sh / (float)(cH[p] > 0 ? cH[p] : 1);
        pk[D + 16 * D + p * D + d] = sw / (float)(cW[p] > 0 ? cW[p] : 1);
      }
    }
    uint8_t* av = axis_valid + (int64_t)z * 24;
    for (int p = 0; p < 8; ++p) {
      av[p] = cT[p] > 0;
      av[8 + p] = cH[p] > 0;
      av[16 + p] = cW[p] > 0;
    }
    float* au = audio + (int64_t)z * 25;
    {
      float cs = 0.0f;
      for (int lt = 0; lt < 8; ++lt) cs += aframe[lt];
      au[0] = cs / fall;
      for (int lt = 0; lt < 8; ++lt) au[1 + lt] = aframe[lt] / (float)(cT[lt] > 0 ? cT[lt] : 1);
      for (int p = 0; p < 8; ++p) {
        float sh = 0.0f, sw = 0.0f;
        for (int lt = 0; lt < 8; ++lt) {
          sh += arow[lt][p];
          sw += acol[lt][p];
        }
        au[9 + p] = sh / (float)(cH[p] > 0 ? cH[p] : 1);
        au[17 + p] = sw / (float)(cW[p] > 0 ? cW[p] : 1);
      }
    }
  }
  free(rowH);
  free(colW);
  free(frame);
}

/* -------------------------------------------------------- shape select */
static const int SHAPES[13][3] = {
    {4, 4, 4}, {8, 2, 4}, {8, 4, 2}, {2, 4, 8}, {2, 8, 4}, {4, 2, 8}, {4, 8, 2},
    {2, 8, 8}, {8, 2, 8}, {8, 8, 2}, {4, 4, 8}, {4, 8, 4}, {8, 4, 4}};

static int ilog2i(int x) { int r = 0; while (x > 1) { x >>= 1; ++r; } return r; }

/* _axis_var, dynamic_block_shape.py:165-178 (masked branch) */
static float axis_var(const float* A, const uint8_t* valid, int D) {
  float n = 0.0f;
  for (int p = 0; p < 8; ++p) n += valid[p] ? 1.0f : 0.0f;
  if (n < 1.0f) n = 1.0f;
  float tot = 0.0f;
  for (int d = 0; d < D; ++d) {
    float s = 0.0f;
    for (int p = 0; p < 8; ++p) if (valid[p]) s += A[p * D + d];
    float mean = s / n;
    float q = 0.0f;
    for (int p = 0; p < 8; ++p) if (valid[p]) { float t = A[p * D + d] - mean; q += t * t; }
    tot += q / n;
  }
  return tot / (float)D;
}

/* _masked_var_1d, dynamic_block_shape.py:181-186 */
static float masked_var8(const float* a, const uint8_t* valid) {
  float n = 0.0f;
  for (int p = 0; p < 8; ++p) n += valid[p] ? 1.0f : 0.0f;
  if (n < 1.0f) n = 1.0f;
  float s = 0.0f;
  for (int p = 0; p < 8; ++p) if (valid[p]) s += a[p];
  float mean = s / n;
  float q = 0.0f;
  for (int p = 0; p < 8; ++p) if (valid[p]) { float t = a[p] - mean; q += t * t; }
  return q / n;
}

/* compute_effective_gradient + select_shapes_{ivpq,penalty},
 * dynamic_block_shape.py:248-355.  method 0 = ivpq, 1 = penalty.
 * has_audio = 0 reproduces audio_norms_thw=None (a_bar = v_hat = 0).
 * g_out [Nz,3] and rho_out [Nz] are optional diagnostics. */
void oracle_shape_select(const float* packed, const uint8_t* axis_valid, const float* audio,
                         int has_audio, int Nz, int D, int method, float lambda_a,
                         float tau_128, float lambda_128, int64_t* shape_ids,
                         float* g_out, float* rho_out) {
  const float EPS = 1e-6f;
  float* rho_raw = (float*)malloc(sizeof(float) * Nz);
  float* aniso = (float*)malloc(sizeof(float) * Nz * 3);
  float* vhat = (float*)malloc(sizeof(float) * Nz * 3);
  float* abar = (float*)malloc(sizeof(float) * Nz);
  for (int z = 0; z < Nz; ++z) {
    const float* pk = packed + (int64_t)z * 25 * D;
    const uint8_t* av = axis_valid + (int64_t)z * 24;
    float s = 0.0f;
    for (int d = 0; d < D; ++d) s += pk[d];
    float gcm = s / (float)D;
    float sv = 0.0f;
    for (int d = 0; d < D; ++d) { float t = pk[d] - gcm; sv += t * t; }
    float spatial = sv / (float)D;
    float npairs = 0.0f;
    uint8_t both[7];
    for (int p = 0; p < 7; ++p) { both[p] = av[p + 1] && av[p]; npairs += both[p] ? 1.0f : 0.0f; }
    if (npairs < 1.0f) npairs = 1.0f;
    float tv = 0.0f;
    for (int d = 0; d < D; ++d) {
      float a = 0.0f;
      for (int p = 0; p < 7; ++p)
        if (both[p]) { float t = pk[D + (p + 1) * D + d] - pk[D + p * D + d]; a += t * t; }
      tv += a / npairs;
    }
    float temporal = tv / (float)D;
    rho_raw[z] = spatial + temporal;
    float vT = axis_var(pk + D, av, D);
    float vH = axis_var(pk + D + 8 * D, av + 8, D);
    float vW = axis_var(pk + D + 16 * D, av + 16, D);
    float asum = (vT + vH) + vW;
    if (asum < EPS) asum = EPS;
    aniso[z * 3 + 0] = vT / asum;
    aniso[z * 3 + 1] = vH / asum;
    aniso[z * 3 + 2] = vW / asum;
    if (has_audio) {
      const float* au = audio + (int64_t)z * 25;
      abar[z] = au[0];
      float aT = masked_var8(au + 1, av);
      float aH = masked_var8(au + 9, av + 8);
      float aW = masked_var8(au + 17, av + 16);
      float den = (aT + aH) + aW;
      if (den < EPS) den = EPS;
      vhat[z * 3 + 0] = aT / den;
      vhat[z * 3 + 1] = aH / den;
      vhat[z * 3 + 2] = aW / den;
    } else {
      abar[z] = 0.0f;
      vhat[z * 3 + 0] = vhat[z * 3 + 1] = vhat[z * 3 + 2] = 0.0f;
    }
  }
  float rmax = rho_raw[0], amax = abar[0];
  for (int z = 1; z < Nz; ++z) {
    if (rho_raw[z] > rmax) rmax = rho_raw[z];
    if (abar[z] > amax) amax = abar[z];
  }
  if (rmax < EPS) rmax = EPS;
  if (amax < EPS) amax = EPS;
  for (int z = 0; z < Nz; ++z) {
    float rho = rho_raw[z] / rmax;
    float an = has_audio ? abar[z] / amax : 0.0f;
    float la = lambda_a * an;
    float g[3];
    for (int d = 0; d < 3; ++d) {
      g[d] = aniso[z * 3 + d] + la * vhat[z * 3 + d];
      if (g[d] < 1e-4f) g[d] = 1e-4f;
    }
    if (g_out) { g_out[z * 3] = g[0]; g_out[z * 3 + 1] = g[1]; g_out[z * 3 + 2] = g[2]; }
    if (rho_out) rho_out[z] = rho;
    const int forbid128 = rho >= tau_128;
    int best = 0;
    float bestv = INFINITY;
    if (method == 0) {
      const float c23 = (float)(-2.0 / 3.0);
      float lr[3];
      for (int d = 0; d < 3; ++d) lr[d] = c23 * oracle_det_log2f(g[d]);
      float sum = (lr[0] + lr[1]) + lr[2];
      float add = (6.0f - sum) / 3.0f;
      float li[3] = {lr[0] + add, lr[1] + add, lr[2] + add};
      for (int c = 0; c < 13; ++c) {
        float dist;
        if (forbid128 && c >= 7) dist = INFINITY;
        else {
          float a0 = (float)ilog2i(SHAPES[c][0]) - li[0];
          float a1 = (float)ilog2i(SHAPES[c][1]) - li[1];
          float a2 = (float)ilog2i(SHAPES[c][2]) - li[2];
          dist = (a0 * a0 + a1 * a1) + a2 * a2;
        }
        if (dist < bestv) { bestv = dist; best = c; }
      }
    } else {
      float bonus = lambda_128 * (1.0f - rho);
      for (int c = 0; c < 13; ++c) {
        float pen;
        if (forbid128 && c >= 7) pen = INFINITY;
        else {
          pen = (g[0] * (float)SHAPES[c][0] + g[1] * (float)SHAPES[c][1]) + g[2] * (float)SHAPES[c][2];
          pen = pen - bonus * (c >= 7 ? 1.0f : 0.0f);
        }
        if (pen < bestv) { bestv = pen; best = c; }
      }
    }
    shape_ids[z] = best;
  }
  free(rho_raw);
  free(aniso);
  free(vhat);
  free(abar);
}

/* -------------------------------------------------------------- layout
 * _precompute_local_orders / _build_rearrange_index / _build_block_tile_maps
 * (dynamic_block_attention.py:21-63, 107-170).
 * src_idx[S], inv_idx[S] (int64), block_of_tile[N_tiles], block_tiles[(N_b+1)*2]
 * (sentinel N_tiles); returns N_b. */
int64_t oracle_layout(const int64_t* shape_ids, int T, int H, int W, int64_t* src_idx,
                      int64_t* inv_idx, int64_t* block_of_tile, int64_t* block_tiles) {
  const int ZT = T / 8, ZH = H / 8, ZW = W / 8;
  const int Nz = ZT * ZH * ZW;
  const int64_t S = (int64_t)T * H * W;
  const int64_t N_tiles = (int64_t)Nz * 8;
  int order[13][512];
  for (int c = 0; c < 13; ++c) {
    const int bt = SHAPES[c][0], bh = SHAPES[c][1], bw = SHAPES[c][2];
    const int bsz = bt * bh * bw, Nh = 8 / bh, Nw = 8 / bw;
    for (int lf = 0; lf < 512; ++lf) {
      int lt = lf / 64, lh = (lf / 8) % 8, lw = lf % 8;
      int blk = ((lt / bt) * Nh + lh / bh) * Nw + lw / bw;
      int off = ((lt % bt) * bh + lh % bh) * bw + lw % bw;
      order[c][blk * bsz + off] = lf;
    }
  }
  int64_t nb = 0;
  for (int z = 0; z < Nz; ++z) {
    const int c = (int)shape_ids[z];
    const int zt = z / (ZH * ZW), zh = (z / ZW) % ZH, zw = z % ZW;
    for (int r = 0; r < 512; ++r) {
      int lf = order[c][r];
      int lt = lf / 64, lh = (lf / 8) % 8, lw = lf % 8;
      int64_t g = ((int64_t)(zt * 8 + lt) * H + (zh * 8 + lh)) * W + (zw * 8 + lw);
      src_idx[(int64_t)z * 512 + r] = g;
    }
    const int bsz = SHAPES[c][0] * SHAPES[c][1] * SHAPES[c][2];
    const int tpb = bsz / 64;
    for (int tl = 0; tl < 8; ++tl) block_of_tile[(int64_t)z * 8 + tl] = nb + tl / tpb;
    nb += 512 / bsz;
  }
  for (int64_t r = 0; r < S; ++r) inv_idx[src_idx[r]] = r;
  for (int64_t b = 0; b < (nb + 1) * 2; ++b) block_tiles[b] = N_tiles;
  for (int64_t j = 0; j < N_tiles; ++j) {
    const int c = (int)shape_ids[j / 8];
    const int tpb = SHAPES[c][0] * SHAPES[c][1] * SHAPES[c][2] / 64;
    block_tiles[block_of_tile[j] * 2 + (j % 8) % tpb] = j;
  }
  return nb;
}

/* ---------------------------------------------------------- selection */
typedef struct { float w; int32_t idx; } wi_t;
static int cmp_wdesc(const void* a, const void* b) {
  const wi_t* x = (const wi_t*)a;
  const wi_t* y = (const wi_t*)b;
  if (x->w > y->w) return -1;
  if (x->w < y->w) return 1;
  return (x->idx < y->idx) ? -1 : (x->idx > y->idx);
}

/* Pooled tile/block means (bsa_interface.py:177-201 masked branch;
 * dynamic_block_attention.py:173-188).  x_re [heads, S, D] bf16 in tile order.
 * tile_mean[j] = (sum_{i valid, sequential} x) / max(count, 1);
 * block_mean[b] = ((0 + m0*c0) + m1*c1) / max(c0 + c1, 1). */
static void pool_blocks(const uint16_t* x_re, int64_t S, int D, const uint8_t* valid_re,
                        int64_t nb, const int64_t* block_tiles, float* out /* [nb, D] */) {
  const int64_t N_tiles = S / 64;
  float* tm = (float*)malloc(sizeof(float) * D);
  for (int64_t b = 0; b < nb; ++b) {
    float cnt = 0.0f;
    for (int d = 0; d < D; ++d) out[b * D + d] = 0.0f;
    for (int p = 0; p < 2; ++p) {
      const int64_t j = block_tiles[b * 2 + p];
      if (j >= N_tiles) continue;
      int c = 0;
      for (int d = 0; d < D; ++d) tm[d] = 0.0f;
      for (int i = 0; i < 64; ++i) {
        const int64_t s = j * 64 + i;
        if (valid_re && !valid_re[s]) continue;
        ++c;
        for (int d = 0; d < D; ++d) tm[d] += bf16_to_f32(x_re[s * D + d]);
      }
      const float fc = (float)c;
      const float den = c > 0 ? fc : 1.0f;
      for (int d = 0; d < D; ++d) out[b * D + d] += (tm[d] / den) * fc;
      cnt += fc;
    }
    const float den = cnt < 1.0f ? 1.0f : cnt;
    for (int d = 0; d < D; ++d) out[b * D + d] = out[b * D + d] / den;
  }
  free(tm);
}

/* Selection sizes of get_select_indices_{cdf_topk,cdf,topk}_from_score
 * (bsa_interface.py:236-304) for nb key blocks: k_topk and the candidate
 * count ub (torch.topk's k). */
static void select_sizes(int mode, double sparsity, double cdf, int64_t nb, int64_t* k_topk_out,
                         int64_t* ub_out) {
  int64_t k_topk = 0, ub = nb;
  if (mode == 0) {
    k_topk = (int64_t)((1.0 - sparsity) * (double)nb);
    if (k_topk < 1) k_topk = 1;
    int64_t u = (int64_t)(cdf * (double)nb) + 1;
    ub = k_topk > u ? k_topk : u;
    if (ub > nb) ub = nb;
  } else if (mode == 1) {
    k_topk = 1;
    ub = (int64_t)(cdf * (double)nb) + 1;
    if (ub > nb) ub = nb;
  } else {
    k_topk = (int64_t)((1.0 - sparsity) * (double)nb);
  }
  *k_topk_out = k_topk;
  *ub_out = ub;
}

/* One row of block scores (score[b], -INFINITY for excluded blocks; clobbered)
 * -> arr sorted by descending key with ties by lower index; returns how many
 * leading entries of arr are selected.  Mode 2 ranks raw scores; modes 0/1
 * rank softmax(score * scale) weights and keep the top-k / cumulative-mass
 * count (cdf_m = round_f32(sum of the top-m weights) with the sum exact in
 * 2^-63 fixed point, as torch's CPU cumsum accumulates in double and rounds
 * each partial sum to float; softmax denominator exact in 2^-50 fixed point,
 * rounded once to float). */
static int64_t select_row(float* score, int64_t nb, int mode, int64_t k_topk, int64_t ub,
                          float scale, float pf, wi_t* arr) {
  if (mode == 2) {
    for (int64_t b = 0; b < nb; ++b) { arr[b].w = score[b]; arr[b].idx = (int32_t)b; }
    qsort(arr, nb, sizeof(wi_t), cmp_wdesc);
    return k_topk;
  }
  float mx = -INFINITY;
  for (int64_t b = 0; b < nb; ++b) {
    float x = score[b] * scale;
    score[b] = x;
    if (x > mx) mx = x;
  }
  uint64_t Z = 0;
  for (int64_t b = 0; b < nb; ++b) {
    float e = oracle_det_expf(score[b] - mx);
    score[b] = e;
    Z += (uint64_t)(e * 0x1p50f);
  }
  const float Zf = (float)Z * 0x1p-50f;
  for (int64_t b = 0; b < nb; ++b) { arr[b].w = score[b] / Zf; arr[b].idx = (int32_t)b; }
  qsort(arr, nb, sizeof(wi_t), cmp_wdesc);
  uint64_t run = 0;
  int64_t cnt_lt = 0;
  for (int64_t m = 0; m < ub; ++m) {
    run += (uint64_t)(arr[m].w * 0x1p63f);
    float cf = (float)run * 0x1p-63f;
    if (cf < pf) ++cnt_lt;
  }
  int64_t n = cnt_lt + 1;
  if (n < k_topk) n = k_topk;
  if (n > nb) n = nb;
  return n < ub ? n : ub;
}

/* Block selection for one head, writing q-tile-major and k-tile-major
 * bitmaps.  mode: 0 = top-k + cdf (get_select_indices_cdf_topk_from_score,
 * bsa_interface.py:284-304), 1 = cdf only (:257-275), 2 = top-k only
 * (:235-248).  Ties are broken by lower block index.
 *
 * Cumulative mass: cdf_m = round_f32(sum of the top-m weights) where the sum
 * is exact in 2^-63 fixed point (torch's CPU cumsum accumulates in double and
 * rounds each partial sum to float).  Softmax denominator: exact in 2^-50
 * fixed point, rounded once to float.
 *
 * bits_q [N_tiles, WQ] u32, bits_k [N_tiles, WQ] u32 with WQ = ceil(N_tiles/32);
 * callers zero them first.  The kept logical-block set per q block is written
 * to sel_blocks [nb, nb] u8 if non-NULL. */
void oracle_block_select(const uint16_t* q_re, const uint16_t* k_re, int heads, int64_t S, int D,
                         const uint8_t* valid_re, int64_t nb, const int64_t* block_tiles,
                         int mode, double sparsity, double cdf, uint32_t* bits_q,
                         uint32_t* bits_k, uint8_t* sel_blocks) {
  const int64_t N_tiles = S / 64;
  const int64_t WQ = (N_tiles + 31) / 32;
  const float scale = (float)(1.0 / sqrt((double)D));
  const float pf = (float)cdf;
  float* qc = (float*)malloc(sizeof(float) * nb * D);
  float* kc = (float*)malloc(sizeof(float) * nb * D);
  float* score = (float*)malloc(sizeof(float) * nb);
  wi_t* arr = (wi_t*)malloc(sizeof(wi_t) * nb);
  int* tile_cnt = (int*)malloc(sizeof(int) * N_tiles);
  uint8_t* bvalid = (uint8_t*)malloc(nb);
  for (int64_t j = 0; j < N_tiles; ++j) {
    int c = 0;
    for (int i = 0; i < 64; ++i) c += valid_re ? (valid_re[j * 64 + i] != 0) : 1;
    tile_cnt[j] = c;
  }
  for (int64_t b = 0; b < nb; ++b) {
    int c = 0;
    for (int p = 0; p < 2; ++p) {
      int64_t j = block_tiles[b * 2 + p];
      if (j < N_tiles) c += tile_cnt[j];
    }
    bvalid[b] = c > 0;
  }
  int64_t k_topk, ub;
  select_sizes(mode, sparsity, cdf, nb, &k_topk, &ub);
  for (int h = 0; h < heads; ++h) {
    pool_blocks(q_re + (int64_t)h * S * D, S, D, valid_re, nb, block_tiles, qc);
    pool_blocks(k_re + (int64_t)h * S * D, S, D, valid_re, nb, block_tiles, kc);
    uint32_t* bq = bits_q + (int64_t)h * N_tiles * WQ;
    uint32_t* bk = bits_k + (int64_t)h * N_tiles * WQ;
    for (int64_t a = 0; a < nb; ++a) {
      for (int64_t b = 0; b < nb; ++b) {
        if (!bvalid[b]) { score[b] = -INFINITY; continue; }
        float acc = 0.0f;
        for (int d = 0; d < D; ++d) acc = fmaf(qc[a * D + d], kc[b * D + d], acc);
        score[b] = acc;
      }
      const int64_t n_eff = select_row(score, nb, mode, k_topk, ub, scale, pf, arr);
      if (sel_blocks) memset(sel_blocks + ((int64_t)h * nb + a) * nb, 0, nb);
      for (int64_t m = 0; m < n_eff; ++m) {
        const int64_t b = arr[m].idx;
        if (sel_blocks) sel_blocks[((int64_t)h * nb + a) * nb + b] = 1;
        for (int p = 0; p < 2; ++p) {
          const int64_t kt = block_tiles[b * 2 + p];
          if (kt >= N_tiles || tile_cnt[kt] == 0) continue;
          for (int pq = 0; pq < 2; ++pq) {
            const int64_t qt = block_tiles[a * 2 + pq];
            if (qt >= N_tiles) continue;
            bq[qt * WQ + kt / 32] |= 1u << (kt % 32);
            bk[kt * WQ + qt / 32] |= 1u << (qt % 32);
          }
        }
      }
    }
  }
  free(qc);
  free(kc);
  free(score);
  free(arr);
  free(tile_cnt);
  free(bvalid);
}

/* Uniform fixed-shape path (_attention_bsa.forward, bsa_interface.py:600-633)
 * on chunk-ordered q_re [heads, Sq, D] / k_re [heads, Sk, D] bf16 whose first
 * seq_q / seq_k rows are real.  Pooling (masked_mean_pooling_compression /
 * mean_pooling_compression, :164-201): chunk mean = sequential fp32 sum over
 * the chunk's valid rows / max(count, 1); q counts the rows with q_valid set
 * (the caller passes the key mask for q and k of one sequence, :609-610, q's
 * own mask for cross attention, or NULL = every row), k the rows with k_valid
 * set (NULL = every real row).  Scores: fmaf chain over d (cal_score,
 * :203-207).  No chunk is excluded from the ranking.  Selected key chunk b
 * covers key tiles [b*tk, b*tk + tk) (tk = chunk_k / 64), tiles without a
 * valid key are dropped; q chunk a's row goes to q tiles [a*tq, a*tq + tq).
 * bits_q [heads, Sq/64, ceil(Sk/2048)], bits_k [heads, Sk/64, ceil(Sq/2048)];
 * sel_chunks [heads, nq, nk] u8 receives the chunk-level selection if non-NULL.
 * Callers zero bits_q / bits_k. */
void oracle_block_select_uniform(const uint16_t* q_re, const uint16_t* k_re, int heads, int64_t Sq,
                                 int64_t Sk, int D, int64_t seq_q, int64_t seq_k, int chunk_q,
                                 int chunk_k, const uint8_t* q_valid, const uint8_t* k_valid,
                                 const float* k_weights, const float* col_scale, int mode,
                                 double sparsity, double cdf, uint32_t* bits_q, uint32_t* bits_k,
                                 uint8_t* sel_chunks) {
  const int64_t NQ_tiles = Sq / 64, NK_tiles = Sk / 64;
  const int64_t WK = (NK_tiles + 31) / 32, WQ = (NQ_tiles + 31) / 32;
  const int64_t nq = seq_q / chunk_q, nk = seq_k / chunk_k;
  const int tq = chunk_q / 64, tk = chunk_k / 64;
  const float scale = (float)(1.0 / sqrt((double)D));
  const float pf = (float)cdf;
  float* qc = (float*)malloc(sizeof(float) * nq * D);
  float* kc = (float*)malloc(sizeof(float) * nk * D);
  float* score = (float*)malloc(sizeof(float) * nk);
  wi_t* arr = (wi_t*)malloc(sizeof(wi_t) * nk);
  int* tile_cnt = (int*)malloc(sizeof(int) * NK_tiles);
  for (int64_t j = 0; j < NK_tiles; ++j) {
    int c = 0;
    for (int i = 0; i < 64; ++i) {
      const int64_t s = j * 64 + i;
      c += s < seq_k && (k_valid ? k_valid[s] != 0 : 1);
    }
    tile_cnt[j] = c;
  }
  int64_t k_topk, ub;
  select_sizes(mode, sparsity, cdf, nk, &k_topk, &ub);
  for (int h = 0; h < heads; ++h) {
    for (int pass = 0; pass < 2; ++pass) {
      const uint16_t* x = pass ? k_re + (int64_t)h * Sk * D : q_re + (int64_t)h * Sq * D;
      const int chunk = pass ? chunk_k : chunk_q;
      const int64_t n = pass ? nk : nq;
      const uint8_t* valid = pass ? k_valid : q_valid;
      float* out = pass ? kc : qc;
      for (int64_t c = 0; c < n; ++c) {
        if (pass && k_weights) { /* Path B: sum of rounded x*w / max(sum w, 1) */
          for (int d = 0; d < D; ++d) {
            float sum = 0.0f, wsum = 0.0f;
            for (int i = 0; i < chunk; ++i) {
              const int64_t s = c * chunk + i;
              const float prod = bf16_to_f32(x[s * D + d]) * k_weights[s];
              sum = sum + prod;
              wsum = wsum + k_weights[s];
            }
            out[c * D + d] = sum / (wsum < 1.0f ? 1.0f : wsum);
          }
          continue;
        }
        int cnt = 0;
        for (int d = 0; d < D; ++d) out[c * D + d] = 0.0f;
        for (int i = 0; i < chunk; ++i) {
          const int64_t s = c * chunk + i;
          if (valid && !valid[s]) continue;
          ++cnt;
          for (int d = 0; d < D; ++d) out[c * D + d] += bf16_to_f32(x[s * D + d]);
        }
        const float den = cnt > 0 ? (float)cnt : 1.0f;
        for (int d = 0; d < D; ++d) out[c * D + d] = out[c * D + d] / den;
      }
    }
    uint32_t* bq = bits_q + (int64_t)h * NQ_tiles * WK;
    uint32_t* bk = bits_k + (int64_t)h * NK_tiles * WQ;
    for (int64_t a = 0; a < nq; ++a) {
      for (int64_t b = 0; b < nk; ++b) {
        float acc = 0.0f;
        for (int d = 0; d < D; ++d) acc = fmaf(qc[a * D + d], kc[b * D + d], acc);
        score[b] = col_scale ? acc * col_scale[b] : acc;
      }
      const int64_t n_eff = select_row(score, nk, mode, k_topk, ub, scale, pf, arr);
      if (sel_chunks) memset(sel_chunks + ((int64_t)h * nq + a) * nk, 0, nk);
      for (int64_t m = 0; m < n_eff; ++m) {
        const int64_t b = arr[m].idx;
        if (sel_chunks) sel_chunks[((int64_t)h * nq + a) * nk + b] = 1;
        for (int p = 0; p < tk; ++p) {
          const int64_t kt = b * tk + p;
          if (tile_cnt[kt] == 0) continue;
          for (int pq = 0; pq < tq; ++pq) {
            const int64_t qt = a * tq + pq;
            bq[qt * WK + kt / 32] |= 1u << (kt % 32);
            bk[kt * WQ + qt / 32] |= 1u << (qt % 32);
          }
        }
      }
    }
  }
  free(qc);
  free(kc);
  free(score);
  free(arr);
  free(tile_cnt);
}

/* ------------------------------------------------------ guided selection
 * Keys in chunk order; k_valid [seq_k] u8 or NULL (= all rows valid).  Same
 * operation order as the CUDA kernels (sequential fp32 sums). */

/* compute_channel_variance_density (bsa_interface.py:973-1062): per chunk of
 * ct frames x (ch*cw) rows, x_avg = (sum over heads) / heads; masked chunk and
 * frame channel means / max(count, 1); spatial = mean_d (cm_d - mean_d cm)^2;
 * temporal = mean_d (sum over pairs of non-empty consecutive frames of the
 * squared frame-mean difference) / max(pairs, 1); rho = combined / max(max, 1e-6). */
void oracle_variance_density(const uint16_t* v_re, int heads, int64_t Sk, int D, int64_t seq_k,
                             int ct, int ch, int cw, const uint8_t* k_valid, float* rho) {
  const int chunk = ct * ch * cw, frame = ch * cw;
  const int64_t n = seq_k / chunk;
  float* cm = (float*)malloc(sizeof(float) * D);
  float* tv = (float*)malloc(sizeof(float) * D);
  for (int64_t c = 0; c < n; ++c) {
    for (int d = 0; d < D; ++d) {
      float csum = 0.0f, fsum = 0.0f, prev = 0.0f, tsum = 0.0f;
      int ccnt = 0, fcnt = 0, pairs = 0, prev_ok = 0;
      for (int i = 0; i < chunk; ++i) {
        const int64_t r = c * chunk + i;
        if (!k_valid || k_valid[r]) {
          float xs = 0.0f;
          for (int h = 0; h < heads; ++h) xs = xs + bf16_to_f32(v_re[((int64_t)h * Sk + r) * D + d]);
          const float xa = xs / (float)heads;
          csum = csum + xa;
          fsum = fsum + xa;
          ++ccnt;
          ++fcnt;
        }
        if ((i + 1) % frame == 0) {
          const float fm = fsum / (fcnt > 0 ? (float)fcnt : 1.0f);
          const int ok = fcnt > 0;
          if (i + 1 > frame && ok && prev_ok) {
            const float df = fm - prev;
            tsum = tsum + df * df;
          }
          if (i + 1 > frame) pairs += ok && prev_ok;
          prev = fm;
          prev_ok = ok;
          fsum = 0.0f;
          fcnt = 0;
        }
      }
      cm[d] = csum / (ccnt > 0 ? (float)ccnt : 1.0f);
      tv[d] = ct > 1 ? tsum / (pairs > 0 ? (float)pairs : 1.0f) : 0.0f;
    }
    float s = 0.0f;
    for (int d = 0; d < D; ++d) s = s + cm[d];
    const float g = s / (float)D;
    float sv = 0.0f, st = 0.0f;
    for (int d = 0; d < D; ++d) {
      const float dv = cm[d] - g;
      sv = sv + dv * dv;
    }
    for (int d = 0; d < D; ++d) st = st + tv[d];
    const float spatial = sv / (float)D;
    const float temporal = ct > 1 ? st / (float)D : 0.0f;
    rho[c] = spatial + temporal;
  }
  float mx = -INFINITY;
  for (int64_t c = 0; c < n; ++c) mx = rho[c] > mx ? rho[c] : mx;
  if (mx < 1e-6f) mx = 1e-6f;
  for (int64_t c = 0; c < n; ++c) rho[c] = rho[c] / mx;
  free(cm);
  free(tv);
}

/* compute_block_audio_saliency (bsa_interface.py:1065-1102): masked chunk means
 * of the norms / max(max, 1e-6). */
void oracle_audio_saliency(const float* norms_re, int64_t seq_k, int chunk, const uint8_t* k_valid,
                           float* out) {
  const int64_t n = seq_k / chunk;
  float mx = -INFINITY;
  for (int64_t c = 0; c < n; ++c) {
    float s = 0.0f;
    int cnt = 0;
    for (int i = 0; i < chunk; ++i) {
      const int64_t r = c * chunk + i;
      if (k_valid && !k_valid[r]) continue;
      s = s + norms_re[r];
      ++cnt;
    }
    out[c] = s / (cnt > 0 ? (float)cnt : 1.0f);
    mx = out[c] > mx ? out[c] : mx;
  }
  if (mx < 1e-6f) mx = 1e-6f;
  for (int64_t c = 0; c < n; ++c) out[c] = out[c] / mx;
}

/* Path B weights (audio_weighted_mean_pooling_compression, bsa_interface.py:944-961):
 * valid rows 1 + lambda * a / max(1e-6, chunk max of valid a), invalid rows 0. */
void oracle_audio_pool_weights(const float* norms_re, int64_t seq_k, int chunk,
                               const uint8_t* k_valid, float lambda_w, float* w) {
  for (int64_t c = 0; c < seq_k / chunk; ++c) {
    float mx = -1e9f;
    for (int i = 0; i < chunk; ++i) {
      const int64_t r = c * chunk + i;
      if ((!k_valid || k_valid[r]) && norms_re[r] > mx) mx = norms_re[r];
    }
    if (mx < 1e-6f) mx = 1e-6f;
    for (int i = 0; i < chunk; ++i) {
      const int64_t r = c * chunk + i;
      w[r] = (!k_valid || k_valid[r]) ? 1.0f + lambda_w * (norms_re[r] / mx) : 0.0f;
    }
  }
}

/* 1 + boost per key chunk (_attention_bsa_audio_guided.forward, bsa_interface.py:
 * 744-764, with the variance term folded into the external modifier as :1467-1470;
 * the variance-only scale 1 + gamma * rho, :1240-1245, is rho alone). */
void oracle_guidance_scale(int64_t n, const float* rho, float var_gamma, const float* sal,
                           float gate, float audio_gamma, const float* modifier, float* scale) {
  const float uni = (float)(1.0 / (double)n);
  for (int64_t c = 0; c < n; ++c) {
    int has_ext = 0;
    float ext = 0.0f;
    if (modifier) {
      ext = modifier[c];
      has_ext = 1;
    }
    if (rho) {
      const float t = var_gamma * rho[c];
      ext = has_ext ? ext + t : t;
      has_ext = 1;
    }
    float boost = 0.0f;
    if (sal) {
      const float a = gate * sal[c];
      const float b = (1.0f - gate) * uni;
      boost = audio_gamma * (a + b);
    }
    if (has_ext) boost = boost + ext;
    scale[c] = 1.0f + boost;
  }
}

/* ---------------------------------------------------- bias rectification */

/* Pooled q / k chunks (fp32 sequential masked means, as oracle_block_select_uniform)
 * and the raw chunk scores (fmaf chain over d).  qc [h, nq, D], kc [h, nk, D],
 * scores [h, nq, nk]. */
void oracle_uniform_pooled(const uint16_t* q_re, const uint16_t* k_re, int heads, int64_t Sq, int64_t Sk,
                           int D, int64_t seq_q, int64_t seq_k, int chunk_q, int chunk_k,
                           const uint8_t* q_valid, const uint8_t* k_valid, float* qc, float* kc,
                           float* scores) {
  const int64_t nq = seq_q / chunk_q, nk = seq_k / chunk_k;
  for (int h = 0; h < heads; ++h) {
    for (int pass = 0; pass < 2; ++pass) {
      const uint16_t* x = pass ? k_re + (int64_t)h * Sk * D : q_re + (int64_t)h * Sq * D;
      const int chunk = pass ? chunk_k : chunk_q;
      const int64_t n = pass ? nk : nq;
      const uint8_t* valid = pass ? k_valid : q_valid;
      float* out = (pass ? kc : qc) + (int64_t)h * n * D;
      for (int64_t c = 0; c < n; ++c) {
        int cnt = 0;
        for (int d = 0; d < D; ++d) out[c * D + d] = 0.0f;
        for (int i = 0; i < chunk; ++i) {
          const int64_t s = c * chunk + i;
          if (valid && !valid[s]) continue;
          ++cnt;
          for (int d = 0; d < D; ++d) out[c * D + d] += bf16_to_f32(x[s * D + d]);
        }
        const float den = cnt > 0 ? (float)cnt : 1.0f;
        for (int d = 0; d < D; ++d) out[c * D + d] = out[c * D + d] / den;
      }
    }
    const float* qh = qc + (int64_t)h * nq * D;
    const float* kh = kc + (int64_t)h * nk * D;
    for (int64_t a = 0; a < nq; ++a)
      for (int64_t b = 0; b < nk; ++b) {
        float acc = 0.0f;
        for (int d = 0; d < D; ++d) acc = fmaf(qh[a * D + d], kh[b * D + d], acc);
        scores[((int64_t)h * nq + a) * nk + b] = acc;
      }
  }
}

/* Sum of 256 strided partials (partial t = sequential sum of x[j], j = t mod 256)
 * combined by halving: p[t] += p[t + s], s = 128, ..., 1. */
static float tree_sum256(const float* p_in) {
  float p[256];
  memcpy(p, p_in, sizeof(p));
  for (int s = 128; s > 0; s >>= 1)
    for (int t = 0; t < s; ++t) p[t] = p[t] + p[t + s];
  return p[0];
}

/* Per head h and q chunk a: A = softmax over valid key chunks of score * sm_scale
 * (deterministic exp), R = max(1 - sum of A over valid unselected chunks, 1e-6),
 * M = variance of A over the valid chunks; sel [h, nq, nk] u8 is the chunk
 * selection, chunk_valid [nk] u8.  nonsel [h, nq, ceil(nk/64)] u64 and a_rect
 * [h, nq, nk] optional.  The operation order of prism_correction_stats. */
void oracle_correction_stats(const float* scores, int heads, int nq, int nk, const uint8_t* sel,
                             const uint8_t* chunk_valid, float sm_scale, float* R, float* M,
                             uint64_t* nonsel, float* a_rect) {
  float* e = (float*)malloc(sizeof(float) * nk);
  const int wn = (nk + 63) / 64;
  float part[256];
  for (int h = 0; h < heads; ++h)
    for (int a = 0; a < nq; ++a) {
      const float* s = scores + ((int64_t)h * nq + a) * nk;
      const uint8_t* sl = sel + ((int64_t)h * nq + a) * nk;
      float mx = -INFINITY;
      int cnt = 0;
      for (int j = 0; j < nk; ++j) {
        e[j] = chunk_valid[j] ? s[j] * sm_scale : -INFINITY;
        if (e[j] > mx) mx = e[j];
        cnt += chunk_valid[j] != 0;
      }
      for (int t = 0; t < 256; ++t) part[t] = 0.0f;
      for (int j = 0; j < nk; ++j) {
        e[j] = e[j] == -INFINITY ? 0.0f : oracle_det_expf(e[j] - mx);
        part[j % 256] = part[j % 256] + e[j];
      }
      const float sum = tree_sum256(part);
      float prect[256], pmean[256];
      for (int t = 0; t < 256; ++t) prect[t] = pmean[t] = 0.0f;
      for (int j = 0; j < nk; ++j) {
        const float A = e[j] / sum;
        e[j] = A;
        const int rect = chunk_valid[j] && !sl[j];
        if (rect) prect[j % 256] = prect[j % 256] + A;
        if (chunk_valid[j]) pmean[j % 256] = pmean[j % 256] + A;
        if (a_rect) a_rect[((int64_t)h * nq + a) * nk + j] = rect ? A : 0.0f;
      }
      const float rsum = tree_sum256(prect);
      const float fn = cnt > 0 ? (float)cnt : 1.0f;
      const float mean = tree_sum256(pmean) / fn;
      for (int t = 0; t < 256; ++t) part[t] = 0.0f;
      for (int j = 0; j < nk; ++j) {
        if (!chunk_valid[j]) continue;
        const float d = e[j] - mean;
        part[j % 256] = part[j % 256] + d * d;
      }
      const float var = tree_sum256(part) / fn;
      const float r = 1.0f - rsum;
      R[(int64_t)h * nq + a] = r < 1e-6f ? 1e-6f : r;
      M[(int64_t)h * nq + a] = var;
      if (nonsel)
        for (int w = 0; w < wn; ++w) {
          uint64_t b = 0;
          for (int i = 0; i < 64; ++i) {
            const int j = w * 64 + i;
            if (j < nk && chunk_valid[j] && !sl[j]) b |= 1ull << i;
          }
          nonsel[((int64_t)h * nq + a) * wn + w] = b;
        }
    }
  free(e);
}
