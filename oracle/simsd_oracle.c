/*
 * simsd_oracle.c - CPU restatement of SimSD's matmul hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the CUDA kernels are
 * compared against; only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline may load it.  The product (libsimsd_b200.so) never calls it.
 *
 * Build: see oracle/Makefile (gcc -O2 -ffp-contract=off: every fp32 operation
 * below is a single IEEE-rounded op, and fmaf() is the correctly rounded fused
 * multiply-add of the C library).
 *
 * Restated reference algorithms (file:line in airevo2/SimSD-release):
 *   oracle_thin_linear         F.linear(x, w, bias), the ground truth of
 *                              kernels/thin_linear_fused.py:265-345 and
 *                              kernels/workspace/thin_linear/CONTRACT.md
 *                              ("Operator + isolated signature"); accumulated
 *                              in fp32 in increasing k.
 *   oracle_thin_linear_silu_mul  SDARMLP's down input silu(gate(x)) * up(x),
 *                              sdar/modeling_sdar.py:113-119.
 *   oracle_route               the synthetic router of
 *                              kernels/workspace/moe_dispatch/build_oracle.py:71-90
 *                              (sigmoid score, top-k, renormalise + 1e-20, routed
 *                              scale) selecting on score + bias; arithmetic fixed
 *                              exactly as the device router documents.
 *   oracle_align               _align, kernels/moe_dispatch_fused.py:93-132.
 *   oracle_moe_dispatch        moe_infer (stock), transcribed at
 *                              kernels/workspace/moe_dispatch/build_oracle.py:34-67,
 *                              with its dtype discipline: every F.linear and the
 *                              silu and the product round to the input dtype, the
 *                              combine runs in fp32 (kernels/moe_dispatch_fused.py:189-192).
 *                              mode 1 keeps gate/up in fp32 until the product
 *                              (the fused kernel's numerics).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- dtypes */
enum { DT_BF16 = 0, DT_F16 = 1, DT_F32 = 2 };

static float bf16_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
  u += 0x7fffu + ((u >> 16) & 1u);                                            /* nearest even */
  return (uint16_t)(u >> 16);
}
static float ld(const void* p, int64_t i, int dt) {
  if (dt == DT_BF16) return bf16_to_f32(((const uint16_t*)p)[i]);
  if (dt == DT_F16) return (float)((const _Float16*)p)[i];
  return ((const float*)p)[i];
}
static void st(void* p, int64_t i, float v, int dt) {
  if (dt == DT_BF16) ((uint16_t*)p)[i] = f32_to_bf16(v);
  else if (dt == DT_F16) ((_Float16*)p)[i] = (_Float16)v;
  else ((float*)p)[i] = v;
}
static float round_to(float v, int dt) {
  if (dt == DT_BF16) return bf16_to_f32(f32_to_bf16(v));
  if (dt == DT_F16) return (float)(_Float16)v;
  return v;
}
static float silu_f(float g) { return g / (1.0f + expf(-g)); }

/* ---------------------------------------------------------------- thin linear */
/* acc[m*N + n] = sum_k x[m,k] w[n,k] (+ bias[n]) in fp32; y = acc rounded to dt. */
void oracle_thin_linear(const void* x, int64_t ldxm, int64_t ldxk, const void* w, int64_t ldwn,
                        int64_t ldwk, const void* bias, int M, int N, int K, int dt, float* acc,
                        void* y) {
  for (int m = 0; m < M; ++m)
    for (int n = 0; n < N; ++n) {
      float s = 0.0f;
      for (int k = 0; k < K; ++k)
        s = fmaf(ld(x, (int64_t)m * ldxm + (int64_t)k * ldxk, dt), ld(w, (int64_t)n * ldwn + (int64_t)k * ldwk, dt), s);
      if (bias) s = s + ld(bias, n, dt);
      if (acc) acc[(int64_t)m * N + n] = s;
      if (y) st(y, (int64_t)m * N + n, s, dt);
    }
}

/* acc = silu(x wg^T) * (x wu^T) with both products in fp32; y = acc rounded. */
void oracle_thin_linear_silu_mul(const void* x, int64_t ldxm, const void* wg, const void* wu,
                                 int64_t ldwn, int M, int I, int K, int dt, float* acc, void* y) {
  for (int m = 0; m < M; ++m)
    for (int i = 0; i < I; ++i) {
      float g = 0.0f, u = 0.0f;
      for (int k = 0; k < K; ++k) {
        const float xv = ld(x, (int64_t)m * ldxm + k, dt);
        g = fmaf(xv, ld(wg, (int64_t)i * ldwn + k, dt), g);
        u = fmaf(xv, ld(wu, (int64_t)i * ldwn + k, dt), u);
      }
      const float h = silu_f(g) * u;
      if (acc) acc[(int64_t)m * I + i] = h;
      if (y) st(y, (int64_t)m * I + i, h, dt);
    }
}

/* ---------------------------------------------------------------- router */
/* exp by Cody-Waite reduction (ln2 = 0.693145751953125 + 1.4286068e-6) and the
 * degree-7 Taylor polynomial of e^r, then two exact power-of-two scalings. */
static float exp_fixed(float x) {
  if (!(x == x)) return x;
  if (x > 88.72283935546875f) return INFINITY;
  if (x < -103.97208404541015625f) return 0.0f;
  const float n = rintf(x * 1.44269502162933349609375f);
  float r = fmaf(n, -0.693145751953125f, x);
  r = fmaf(n, -1.428606765330187045037746429443359375e-06f, r);
  float q = 1.98412701138295233249664306640625e-04f;
  q = fmaf(q, r, 1.3888889225199818611145019531250e-03f);
  q = fmaf(q, r, 8.3333337679505348205566406250000e-03f);
  q = fmaf(q, r, 4.1666667908430099487304687500000e-02f);
  q = fmaf(q, r, 1.6666667163372039794921875000000e-01f);
  q = fmaf(q, r, 0.5f);
  q = fmaf(q, r, 1.0f);
  q = fmaf(q, r, 1.0f);
  const int ni = (int)n;
  const int n1 = ni >> 1;
  const int n2 = ni - n1;
  uint32_t b1 = (uint32_t)(n1 + 127) << 23, b2 = (uint32_t)(n2 + 127) << 23;
  float s1, s2;
  memcpy(&s1, &b1, 4);
  memcpy(&s2, &b2, 4);
  q = q * s1;
  q = q * s2;
  return q;
}

/* logit[t,e]: 32 lane partials (lane l sums the 8-element chunks l, l+32, ... in
 * increasing element order with fmaf), then the xor butterfly 16,8,4,2,1. */
static float route_logit(const void* x, int64_t xo, int xdt, const void* w, int64_t wo, int wdt,
                         int H) {
  float v[32];
  const int nch = (H + 7) / 8;
  for (int l = 0; l < 32; ++l) {
    float a = 0.0f;
    for (int c = l; c < nch; c += 32)
      for (int i = 0; i < 8 && c * 8 + i < H; ++i)
        a = fmaf(ld(x, xo + c * 8 + i, xdt), ld(w, wo + c * 8 + i, wdt), a);
    v[l] = a;
  }
  for (int m = 16; m > 0; m >>= 1) {
    float nv[32];
    for (int l = 0; l < 32; ++l) nv[l] = v[l] + v[l ^ m];
    memcpy(v, nv, sizeof(v));
  }
  return v[0];
}

void oracle_route(const void* x, int64_t ldx, int xdt, const void* w, int64_t ldw, int wdt,
                  const float* bias, int T, int H, int E, int k, int renorm, float scale,
                  int64_t* ids, float* wts, float* logits) {
  float* score = (float*)malloc(sizeof(float) * E);
  float* choice = (float*)malloc(sizeof(float) * E);
  char* taken = (char*)malloc(E);
  for (int t = 0; t < T; ++t) {
    for (int e = 0; e < E; ++e) {
      const float lg = route_logit(x, (int64_t)t * ldx, xdt, w, (int64_t)e * ldw, wdt, H);
      if (logits) logits[(int64_t)t * E + e] = lg;
      score[e] = 1.0f / (1.0f + exp_fixed(-lg));
      choice[e] = bias ? score[e] + bias[e] : score[e];
      taken[e] = 0;
    }
    float sel[64];
    for (int j = 0; j < k; ++j) {
      int be = -1;
      float bb = 0.0f;
      for (int e = 0; e < E; ++e) {
        if (taken[e]) continue;
        float v = choice[e];
        if (v != v) v = -INFINITY;
        if (be < 0 || v > bb) { bb = v; be = e; }
      }
      if (be >= 0) taken[be] = 1;
      ids[(int64_t)t * k + j] = be;
      sel[j] = be >= 0 ? score[be] : 0.0f;
    }
    const int norm = renorm && k > 1;
    float denom = 1.0f;
    if (norm) {
      float s = sel[0];
      for (int j = 1; j < k; ++j) s = s + sel[j];
      denom = s + 1e-20f;
    }
    for (int j = 0; j < k; ++j) {
      float v = sel[j];
      if (norm) v = v / denom;
      wts[(int64_t)t * k + j] = v * scale;
    }
  }
  free(score);
  free(choice);
  free(taken);
}

/* ---------------------------------------------------------------- align */
/* counts, offsets (exclusive prefix), stable argsort of ids by value, its inverse,
 * and the reference's padded layout: groups padded to block_m rows (-1 = pad),
 * tile_expert[t] = number of padded group ends <= t*block_m.  Returns 0, or -1
 * if an id is out of range (that slot maps to row -1). */
int oracle_align(const int64_t* ids, int S, int E, int32_t* counts, int32_t* offsets,
                 int32_t* sorted_slots, int32_t* slot_to_row, int block_m, int num_tiles,
                 int32_t* slots_padded, int32_t* tile_expert) {
  int bad = 0;
  for (int e = 0; e < E; ++e) counts[e] = 0;
  for (int s = 0; s < S; ++s) {
    if (ids[s] < 0 || ids[s] >= E) { bad = 1; continue; }
    counts[ids[s]]++;
  }
  offsets[0] = 0;
  for (int e = 0; e < E; ++e) offsets[e + 1] = offsets[e] + counts[e];
  int32_t* fill = (int32_t*)malloc(sizeof(int32_t) * (E + 1));
  for (int e = 0; e <= E; ++e) fill[e] = offsets[e];
  for (int s = 0; s < S; ++s) {
    if (ids[s] < 0 || ids[s] >= E) { slot_to_row[s] = -1; continue; }
    const int row = fill[ids[s]]++;
    sorted_slots[row] = s;
    slot_to_row[s] = row;
  }
  if (slots_padded) {
    int64_t* pad_end = (int64_t*)malloc(sizeof(int64_t) * (E + 1));
    pad_end[0] = 0;
    for (int e = 0; e < E; ++e) pad_end[e + 1] = pad_end[e] + ((counts[e] + block_m - 1) / block_m) * (int64_t)block_m;
    const int64_t npad = (int64_t)num_tiles * block_m;
    for (int64_t i = 0; i < npad; ++i) slots_padded[i] = -1;
    for (int e = 0; e < E; ++e)
      for (int r = 0; r < counts[e]; ++r) {
        const int64_t dst = pad_end[e] + r;
        if (dst < npad) slots_padded[dst] = sorted_slots[offsets[e] + r];
        else bad = 1;
      }
    for (int t = 0; t < num_tiles; ++t) {
      const int64_t v = (int64_t)t * block_m;
      int c = 0;
      while (c < E && pad_end[c + 1] <= v) ++c;
      tile_expert[t] = c;
    }
    free(pad_end);
  }
  free(fill);
  return bad ? -1 : 0;
}

/* ---------------------------------------------------------------- MoE dispatch */
/* out[t] = round( sum_j fl(fp32(y_{t,j}) * w[t,j]) ) in increasing j, where
 *   mode 0 (stock moe_infer): g = rnd(x.wg), u = rnd(x.wu), h = rnd(rnd(silu(g)) * u),
 *   mode 1 (fused numerics):  h = rnd(silu(x.wg) * (x.wu)) with fp32 products,
 * and y = rnd(h . wd); all dot products accumulate in fp32 in increasing index.
 * `add` (T,H) or NULL: out = rnd(rnd(sum) + add).  acc (T,H) fp32 or NULL: the
 * unrounded combine. */
void oracle_moe_dispatch(const void* x, const int64_t* ids, const float* w, const void* wg,
                         const void* wu, const void* wd, const void* add, int T, int k, int E,
                         int H, int I, int dt, int mode, float* acc, void* out) {
  float* h = (float*)malloc(sizeof(float) * I);
  float* y = (float*)malloc(sizeof(float) * H);
  float* sum = (float*)malloc(sizeof(float) * H);
  for (int t = 0; t < T; ++t) {
    for (int c = 0; c < H; ++c) sum[c] = 0.0f;
    for (int j = 0; j < k; ++j) {
      const int64_t e = ids[(int64_t)t * k + j];
      if (e < 0 || e >= E) continue;
      for (int i = 0; i < I; ++i) {
        float g = 0.0f, u = 0.0f;
        for (int c = 0; c < H; ++c) {
          const float xv = ld(x, (int64_t)t * H + c, dt);
          g = fmaf(xv, ld(wg, (e * I + i) * (int64_t)H + c, dt), g);
          u = fmaf(xv, ld(wu, (e * I + i) * (int64_t)H + c, dt), u);
        }
        if (mode == 0) {
          g = round_to(g, dt);
          u = round_to(u, dt);
          h[i] = round_to(round_to(silu_f(g), dt) * u, dt);
        } else {
          h[i] = round_to(silu_f(g) * u, dt);
        }
      }
      for (int c = 0; c < H; ++c) {
        float s = 0.0f;
        for (int i = 0; i < I; ++i) s = fmaf(h[i], ld(wd, (e * H + c) * (int64_t)I + i, dt), s);
        y[c] = round_to(s, dt);
      }
      const float wt = w[(int64_t)t * k + j];
      for (int c = 0; c < H; ++c) sum[c] = sum[c] + y[c] * wt;
    }
    for (int c = 0; c < H; ++c) {
      float v = sum[c];
      if (acc) acc[(int64_t)t * H + c] = v;
      if (add) v = round_to(v, dt) + ld(add, (int64_t)t * H + c, dt);
      st(out, (int64_t)t * H + c, v, dt);
    }
  }
  free(h);
  free(y);
  free(sum);
}
