/*
 * TEST INFRASTRUCTURE ONLY (oracle). A plain-C restatement of malkin's CPU verify path, used by tests/,
 * __graft_entry__.smoke() and bench.py's CPU baseline as the checker. The product (malkin_b200) never links or
 * calls it. Every function cites the reference file:line it follows (kekzl/malkin v0.2.0, src/...).
 *
 * Pinned by tests/test_oracle.py against oracle/_ref (malkin's own sources compiled unchanged) and against the
 * committed golden fixtures under tests/golden/ (made by tests/golden/make_golden.py from oracle/_ref):
 *   bit-exact:  quantize_row_q8 / BlockQ8, quantize_i8, dequantize_row, integer block dots, matmul through the
 *               compact panel kernels, attention, and the full forward's logits: every float operation of malkin's
 *               path is restated in malkin's order, including the 16-lane AVX-512 partial sums and their horizontal
 *               reduction (reduce16) and the fused multiply-adds g++ forms from model.cpp / quant.cpp scalar code
 *               (FMA contraction is on for C++ at -O2 -march=x86-64-v4), so logits are bit-identical;
 *   decisions:  accept walks and sampler decisions on identical logits.
 * Built with -ffp-contract=off so every a*b+c below is two roundings unless written as fmaf.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define ORC_F32 0
#define ORC_F16 1
#define ORC_Q8_0 8
#define ORC_Q4_K 12
#define ORC_Q6_K 14

typedef struct {
  float d;
  int16_t s[2];
  int8_t qs[32];
} orc_block_q8; /* quant.h:11-16 */

/* ---------------- scalars ---------------- */

static float f16(const uint8_t* p) {
  const uint16_t h = (uint16_t)(p[0] | (p[1] << 8));
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  const int exp = (h >> 10) & 31;
  const uint32_t man = h & 1023;
  uint32_t bits;
  if (exp == 0) {
    const float v = ldexpf((float)man, -24);
    return sign ? -v : v;
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((uint32_t)(exp - 15 + 127) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

float orc_fp16_to_fp32(uint16_t h) {
  uint8_t b[2] = {(uint8_t)(h & 0xFF), (uint8_t)(h >> 8)};
  return f16(b);
}

/* round half to even, as vcvtps2dq under the default MXCSR and lrintf */
static int rne(float x) { return (int)lrintf(x); }

/* e^x of malkin's softmax / SiLU (kernels_avx512.cpp:186-203): clamp at -87, Cody-Waite with ln 2 in two parts,
 * degree-6 Taylor in Horner form with fused multiply-adds, scale by 2^n. */
static float exp_malkin(float x) {
  if (x < -87.0f) x = -87.0f;
  const float n = rintf(x * 1.44269504088896341f);
  float r = fmaf(-n, 0.693145751953125f, x);
  r = fmaf(-n, 1.42860682030941723e-6f, r);
  float p = 1.0f / 720.0f;
  p = fmaf(p, r, 1.0f / 120.0f);
  p = fmaf(p, r, 1.0f / 24.0f);
  p = fmaf(p, r, 1.0f / 6.0f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  return ldexpf(p, (int)n);
}

/* ---------------- quantization (kernels_avx512.cpp:66-80, quant.cpp:134-140) ---------------- */

void orc_quantize_row_q8(const float* x, orc_block_q8* y, int64_t k) {
  for (int64_t i = 0; i < k / 32; ++i, x += 32) {
    float amax = 0.0f;
    for (int l = 0; l < 32; ++l) amax = fmaxf(amax, fabsf(x[l]));
    const float d = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    int s0 = 0, s1 = 0;
    for (int l = 0; l < 32; ++l) {
      const int q = rne(x[l] * id);
      y[i].qs[l] = (int8_t)(q > 127 ? 127 : q < -128 ? -128 : q);
      if (l < 16)
        s0 += q;
      else
        s1 += q;
    }
    y[i].d = d;
    y[i].s[0] = (int16_t)s0;
    y[i].s[1] = (int16_t)s1;
  }
}

float orc_quantize_i8(const float* x, int n, int8_t* q) {
  float amax = 0.0f;
  for (int i = 0; i < n; ++i) amax = fmaxf(amax, fabsf(x[i]));
  const float d = amax / 127.0f, id = d != 0.0f ? 1.0f / d : 0.0f;
  for (int i = 0; i < n; ++i) q[i] = (int8_t)lrintf(x[i] * id);
  return d;
}

/* ---------------- GGUF formats (quant.cpp:70-169, kernels.h:18-26) ---------------- */

static void scale_min_k4(int j, const uint8_t* q, int* sc, int* m) {
  if (j < 4) {
    *sc = q[j] & 63;
    *m = q[j + 4] & 63;
  } else {
    *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
    *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

static int q6_at(const uint8_t* s, int k) {
  const int n = k / 128, rem = k % 128, c = rem / 32, l = rem % 32;
  const uint8_t lo = s[64 * n + l + (c & 1) * 32];
  const int nib = c >= 2 ? lo >> 4 : lo & 0xF;
  return nib | (((s[128 + 32 * n + l] >> (2 * c)) & 3) << 4);
}

size_t orc_row_bytes(int type, int64_t k) {
  switch (type) {
    case ORC_F32:
      return (size_t)k * 4;
    case ORC_F16:
      return (size_t)k * 2;
    case ORC_Q8_0:
      return (size_t)(k / 32) * 34;
    case ORC_Q4_K:
      return (size_t)(k / 256) * 144;
    case ORC_Q6_K:
      return (size_t)(k / 256) * 210;
    default:
      return 0;
  }
}

int orc_dequantize_row(int type, const uint8_t* b, float* y, int64_t k) {
  switch (type) {
    case ORC_F32:
      memcpy(y, b, (size_t)k * 4);
      return 0;
    case ORC_F16:
      for (int64_t i = 0; i < k; ++i) y[i] = f16(b + 2 * i);
      return 0;
    case ORC_Q8_0:
      for (int64_t i = 0; i < k / 32; ++i, b += 34) {
        const float d = f16(b);
        for (int l = 0; l < 32; ++l) y[i * 32 + l] = d * (float)(int8_t)b[2 + l];
      }
      return 0;
    case ORC_Q4_K:
      for (int64_t i = 0; i < k / 256; ++i, b += 144) {
        const float d = f16(b), dmin = f16(b + 2);
        const uint8_t* q = b + 16;
        for (int j = 0; j < 4; ++j, q += 32) {
          int s0, m0, s1, m1;
          scale_min_k4(2 * j, b + 4, &s0, &m0);
          scale_min_k4(2 * j + 1, b + 4, &s1, &m1);
          /* d * s * q - dmin * m as g++ contracts it: fma(q, d * s, -(dmin * m)) */
          for (int l = 0; l < 32; ++l) *y++ = fmaf((float)(q[l] & 0xF), d * (float)s0, -(dmin * (float)m0));
          for (int l = 0; l < 32; ++l) *y++ = fmaf((float)(q[l] >> 4), d * (float)s1, -(dmin * (float)m1));
        }
      }
      return 0;
    case ORC_Q6_K:
      for (int64_t i = 0; i < k / 256; ++i, b += 210) {
        const float d = f16(b + 208);
        const int8_t* sc = (const int8_t*)(b + 192);
        for (int p = 0; p < 256; ++p) y[p] = d * (float)sc[p / 16] * (float)(q6_at(b, p) - 32);
        y += 256;
      }
      return 0;
    default:
      return -1;
  }
}

/* ---------------- GEMM: the compact panel kernels' arithmetic (gemm_avx512.cpp:67-205) ---------------- */

/* Exact integer dot of block b (32 values; Q6_K: 16-value half h) of weight row w with activation block x. */
static int dot_q8_0_block(const uint8_t* w, int64_t b, const orc_block_q8* x) {
  const uint8_t* blk = w + b * 34 + 2;
  int s = 0;
  for (int l = 0; l < 32; ++l) s += (int8_t)blk[l] * x->qs[l];
  return s;
}

static int dot_q4_k_block(const uint8_t* w, int64_t b, const orc_block_q8* x) {
  const uint8_t* sb = w + (b / 8) * 144;
  const int j = (int)(b % 8);
  int s = 0;
  for (int l = 0; l < 32; ++l) {
    const uint8_t q8 = sb[16 + 32 * (j / 2) + l];
    s += ((j & 1) ? q8 >> 4 : q8 & 0xF) * x->qs[l];
  }
  return s;
}

/* Q6_K half h of 32-block b: sum (q - 32) * x over 16 values (= ai - 32 * s[h], gemm_avx512.cpp:193-199) */
static int dot_q6_k_half(const uint8_t* w, int64_t b, int h, const orc_block_q8* x) {
  const uint8_t* sb = w + (b / 8) * 210;
  const int base = (int)(b % 8) * 32 + 16 * h;
  int s = 0;
  for (int l = 0; l < 16; ++l) s += (q6_at(sb, base + l) - 32) * x->qs[16 * h + l];
  return s;
}

/* out[(r * n + t) * nblk + b] (Q6_K: nblk = 2 * cols / 32 halves) */
void orc_block_dots(int type, const uint8_t* w, int64_t rows, int64_t cols, const orc_block_q8* xq, int n,
                    int32_t* out) {
  const size_t rb = orc_row_bytes(type, cols);
  const int64_t nb = cols / 32;
  const int64_t nblk = type == ORC_Q6_K ? 2 * nb : nb;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const uint8_t* wr = w + (size_t)r * rb;
    for (int t = 0; t < n; ++t) {
      int32_t* o = out + ((size_t)r * n + t) * nblk;
      for (int64_t b = 0; b < nb; ++b) {
        const orc_block_q8* x = xq + (size_t)t * nb + b;
        if (type == ORC_Q8_0) {
          o[b] = dot_q8_0_block(wr, b, x);
        } else if (type == ORC_Q4_K) {
          o[b] = dot_q4_k_block(wr, b, x);
        } else {
          o[2 * b] = dot_q6_k_half(wr, b, 0, x);
          o[2 * b + 1] = dot_q6_k_half(wr, b, 1, x);
        }
      }
    }
  }
}

/* y[t * rows + r] = W[r] . x[t], activations as BlockQ8: per (row, token) one float accumulator over the blocks in
 * order, acc = fma(float(dot), d_w * d_x, acc) (Q8_0, gemm_avx512.cpp:91-98); Q4_K: then acc = fma(-(dmin*m), d_x *
 * float(s0+s1), acc) (:142-150); Q6_K: per 16-half, acc = fma(float(dot), (d*sc) * d_x, acc) (:193-199). */
void orc_matmul_q8(int type, const uint8_t* w, int64_t rows, int64_t cols, const orc_block_q8* xq, int n, float* y) {
  const size_t rb = orc_row_bytes(type, cols);
  const int64_t nb = cols / 32;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const uint8_t* wr = w + (size_t)r * rb;
    for (int t = 0; t < n; ++t) {
      const orc_block_q8* xr = xq + (size_t)t * nb;
      float acc = 0.0f;
      for (int64_t b = 0; b < nb; ++b) {
        const orc_block_q8* x = xr + b;
        if (type == ORC_Q8_0) {
          const float dw = f16(wr + b * 34);
          acc = fmaf((float)dot_q8_0_block(wr, b, x), dw * x->d, acc);
        } else if (type == ORC_Q4_K) {
          const uint8_t* sb = wr + (b / 8) * 144;
          int sc, m;
          scale_min_k4((int)(b % 8), sb + 4, &sc, &m);
          const float scf = f16(sb) * (float)sc, mnf = f16(sb + 2) * (float)m;
          const float dsx = x->d * (float)(x->s[0] + x->s[1]);
          acc = fmaf((float)dot_q4_k_block(wr, b, x), scf * x->d, acc);
          acc = fmaf(-mnf, dsx, acc);
        } else {
          const uint8_t* sb = wr + (b / 8) * 210;
          const float d = f16(sb + 208);
          const int8_t* sc = (const int8_t*)(sb + 192);
          for (int h = 0; h < 2; ++h) {
            const float dsc = d * (float)sc[(b % 8) * 2 + h];
            acc = fmaf((float)dot_q6_k_half(wr, b, h, x), dsc * x->d, acc);
          }
        }
      }
      y[(size_t)t * rows + r] = acc;
    }
  }
}

void orc_matmul(int type, const uint8_t* w, int64_t rows, int64_t cols, const float* x, int n, float* y) {
  const int64_t nb = cols / 32;
  orc_block_q8* xq = (orc_block_q8*)malloc(sizeof(orc_block_q8) * (size_t)(n * nb));
  for (int t = 0; t < n; ++t) orc_quantize_row_q8(x + (size_t)t * cols, xq + (size_t)t * nb, cols);
  orc_matmul_q8(type, w, rows, cols, xq, n, y);
  free(xq);
}

/* ---------------- small ops ---------------- */

/* The 16-lane horizontal sum of an AVX-512 register (_mm512_reduce_add_ps): lanes i and i + 8 first, then i and
 * i + 4, then i and i + 2, then lanes 0 and 1 (IEEE addition is commutative, so operand order does not matter). */
static float reduce16(const float* a) {
  float b[8], c[4];
  for (int i = 0; i < 8; ++i) b[i] = a[i + 8] + a[i];
  for (int i = 0; i < 4; ++i) c[i] = b[i + 4] + b[i];
  return (c[0] + c[2]) + (c[1] + c[3]);
}

/* kern::dot_f32 (kernels_avx512.cpp:82-89): 16 lanes, lane l accumulating elements l, l + 16, ... by fma in order,
 * then reduce16; a scalar tail for n % 16. */
static float dot_f32_16(const float* w, const float* x, int n) {
  float acc[16] = {0};
  int i = 0;
  for (; i + 16 <= n; i += 16)
    for (int l = 0; l < 16; ++l) acc[l] = fmaf(w[i + l], x[i + l], acc[l]);
  float s = reduce16(acc);
  for (; i < n; ++i) s += w[i] * x[i];
  return s;
}

/* rmsnorm (model.cpp:46-49): s = 1 / sqrt(dot_f32(x, x) / n + eps), y = x * s * w */
static void rmsnorm(float* y, const float* x, const float* w, int n, float eps) {
  const float s = 1.0f / sqrtf(dot_f32_16(x, x, n) / (float)n + eps);
  for (int i = 0; i < n; ++i) y[i] = x[i] * s * w[i];
}

/* kern::silu_mul (kernels_avx512.cpp:271-280) */
void orc_silu_mul(int64_t n, float* g, const float* u) {
  for (int64_t i = 0; i < n; ++i) g[i] = g[i] / (1.0f + exp_malkin(0.0f - g[i])) * u[i];
}

/* kern::attend_gqa (kernels_avx512.cpp:229-307): one token, the G heads of one KV head. Keys 0..n-1 then extra[].
 * k / v: head row 0 of int8 values, rows `stride` bytes apart; scales at ks[row] / vs[row]. */
void orc_attend(const float* q, int G, int D, const int8_t* k, const int8_t* v, const float* ks, const float* vs,
                int64_t stride, int n, const int* extra, int ne, float scale, float* out) {
  const int nk = n + ne;
  float* s = (float*)malloc(sizeof(float) * (size_t)nk);
  for (int h = 0; h < G; ++h) {
    float mx = -INFINITY;
    for (int j = 0; j < nk; ++j) {
      const int64_t row = j < n ? j : extra[j - n];
      const int8_t* kr = k + row * stride;
      /* attend_t's score: 16 lanes over d, the first product a multiply, then fma in d order; reduce16 */
      float acc[16];
      for (int l = 0; l < 16; ++l) acc[l] = q[h * D + l] * (float)kr[l];
      for (int d0 = 16; d0 < D; d0 += 16)
        for (int l = 0; l < 16; ++l) acc[l] = fmaf(q[h * D + d0 + l], (float)kr[d0 + l], acc[l]);
      s[j] = reduce16(acc) * (ks[row] * scale);
      if (s[j] > mx) mx = s[j];
    }
    /* softmax_inplace (kernels_avx512.cpp:205-226): e = exp(s - max); sums in 16 lanes (key j in lane j % 16) */
    float sum16[16] = {0};
    for (int j = 0; j < nk; ++j) {
      s[j] = exp_malkin(s[j] - mx);
      sum16[j % 16] += s[j];
    }
    const float inv = 1.0f / reduce16(sum16);
    for (int d = 0; d < D; ++d) out[h * D + d] = 0.0f;
    for (int j = 0; j < nk; ++j) {
      const int64_t row = j < n ? j : extra[j - n];
      const float pv = s[j] * vs[row];
      const int8_t* vr = v + row * stride;
      for (int d = 0; d < D; ++d) out[h * D + d] = fmaf(pv, (float)vr[d], out[h * D + d]);
    }
    for (int d = 0; d < D; ++d) out[h * D + d] *= inv;
  }
  free(s);
}

/* ---------------- GGUF v3 (gguf.cpp:205-249) ---------------- */

typedef struct {
  char name[96];
  int type;
  int64_t ne[4];
  int nd;
  const uint8_t* data;
} orc_tensor;

typedef struct orc_model {
  uint8_t* file;
  size_t size;
  int n_tensors;
  orc_tensor* t;
  int n_layer, n_embd, n_ff, n_head, n_head_kv, head_dim, n_vocab, n_ctx, n_seq;
  float rope_base, rms_eps;
  const orc_tensor *tok, *out, *onorm;
  const orc_tensor** L; /* per layer: attn_norm ffn_norm q_norm k_norm q k v o gate up down */
  int8_t *kc, *vc;      /* [layer][kvh][seq * n_ctx + pos][D] */
  float *ksc, *vsc;     /* [layer][kvh][seq * n_ctx + pos] */
  float* inv_freq;
} orc_model;

typedef struct {
  const uint8_t* p;
  const uint8_t* end;
} cur_t;

static int rd(cur_t* c, void* dst, size_t n) {
  if ((size_t)(c->end - c->p) < n) return -1;
  memcpy(dst, c->p, n);
  c->p += n;
  return 0;
}

static uint64_t rd64(cur_t* c) {
  uint64_t v = 0;
  rd(c, &v, 8);
  return v;
}
static uint32_t rd32(cur_t* c) {
  uint32_t v = 0;
  rd(c, &v, 4);
  return v;
}

static size_t scalar_size(uint32_t t) {
  static const size_t sz[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
  return t < 13 ? sz[t] : 0;
}

static int64_t rd_int(cur_t* c, uint32_t t) {
  switch (t) {
    case 0: { uint8_t v = 0; rd(c, &v, 1); return v; }
    case 1: { int8_t v = 0; rd(c, &v, 1); return v; }
    case 2: { uint16_t v = 0; rd(c, &v, 2); return v; }
    case 3: { int16_t v = 0; rd(c, &v, 2); return v; }
    case 4: { uint32_t v = 0; rd(c, &v, 4); return v; }
    case 5: { int32_t v = 0; rd(c, &v, 4); return v; }
    case 10: { uint64_t v = 0; rd(c, &v, 8); return (int64_t)v; }
    case 11: { int64_t v = 0; rd(c, &v, 8); return v; }
    default: return 0;
  }
}

static const orc_tensor* find_t(const orc_model* m, const char* name) {
  for (int i = 0; i < m->n_tensors; ++i)
    if (strcmp(m->t[i].name, name) == 0) return &m->t[i];
  return NULL;
}

static int64_t t_rows(const orc_tensor* t) {
  int64_t n = 1;
  for (int d = 1; d < t->nd; ++d) n *= t->ne[d];
  return n;
}

void orc_model_close(orc_model* m) {
  if (!m) return;
  free(m->file);
  free(m->t);
  free(m->L);
  free(m->kc);
  free(m->vc);
  free(m->ksc);
  free(m->vsc);
  free(m->inv_freq);
  free(m);
}

/* GgufFile + read_config + Model::Model + alloc_kv (model.cpp:78-152, 197-202); NULL on error. */
orc_model* orc_model_open(const char* path, int n_ctx, int n_seq) {
  FILE* f = fopen(path, "rb");
  if (!f) return NULL;
  fseek(f, 0, SEEK_END);
  const long sz = ftell(f);
  fseek(f, 0, SEEK_SET);
  orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
  m->file = (uint8_t*)malloc((size_t)sz);
  m->size = (size_t)sz;
  if (fread(m->file, 1, (size_t)sz, f) != (size_t)sz) {
    fclose(f);
    orc_model_close(m);
    return NULL;
  }
  fclose(f);
  cur_t c = {m->file, m->file + sz};
  if (rd32(&c) != 0x46554747u || rd32(&c) < 3) {
    orc_model_close(m);
    return NULL;
  }
  const uint64_t nt = rd64(&c), nkv = rd64(&c);
  int64_t align = 32, n_vocab_tokens = 0;
  int have_kv = 0, have_hd = 0;
  m->rope_base = 10000.0f;
  m->rms_eps = 1e-6f;
  for (uint64_t i = 0; i < nkv; ++i) {
    const uint64_t kl = rd64(&c);
    char key[256] = {0};
    rd(&c, key, kl < 255 ? kl : 255);
    if (kl >= 255) c.p += kl - 255;
    const uint32_t t = rd32(&c);
    if (t == 8) { /* string */
      const uint64_t n = rd64(&c);
      c.p += n;
    } else if (t == 9) { /* array */
      const uint32_t et = rd32(&c);
      const uint64_t n = rd64(&c);
      if (strcmp(key, "tokenizer.ggml.tokens") == 0) n_vocab_tokens = (int64_t)n;
      if (et == 8) {
        for (uint64_t j = 0; j < n; ++j) c.p += rd64(&c);
      } else {
        c.p += scalar_size(et) * n;
      }
    } else if (t == 6 || t == 12) { /* float */
      double v;
      if (t == 6) {
        float fv;
        rd(&c, &fv, 4);
        v = fv;
      } else {
        rd(&c, &v, 8);
      }
      if (strcmp(key, "qwen3.rope.freq_base") == 0) m->rope_base = (float)v;
      if (strcmp(key, "qwen3.attention.layer_norm_rms_epsilon") == 0) m->rms_eps = (float)v;
    } else {
      const int64_t v = t == 7 ? (int64_t)(*c.p++ != 0) : rd_int(&c, t);
      if (strcmp(key, "qwen3.block_count") == 0) m->n_layer = (int)v;
      if (strcmp(key, "qwen3.embedding_length") == 0) m->n_embd = (int)v;
      if (strcmp(key, "qwen3.feed_forward_length") == 0) m->n_ff = (int)v;
      if (strcmp(key, "qwen3.attention.head_count") == 0) m->n_head = (int)v;
      if (strcmp(key, "qwen3.attention.head_count_kv") == 0) m->n_head_kv = (int)v, have_kv = 1;
      if (strcmp(key, "qwen3.attention.key_length") == 0) m->head_dim = (int)v, have_hd = 1;
      if (strcmp(key, "general.alignment") == 0) align = v;
    }
  }
  (void)n_vocab_tokens;
  if (!have_kv) m->n_head_kv = m->n_head;
  if (!have_hd) m->head_dim = m->n_embd / m->n_head;
  m->n_tensors = (int)nt;
  m->t = (orc_tensor*)calloc(nt, sizeof(orc_tensor));
  uint64_t* off = (uint64_t*)calloc(nt, 8);
  for (uint64_t i = 0; i < nt; ++i) {
    const uint64_t nl = rd64(&c);
    rd(&c, m->t[i].name, nl < 95 ? nl : 95);
    if (nl >= 95) c.p += nl - 95;
    m->t[i].nd = (int)rd32(&c);
    for (int d = 0; d < m->t[i].nd; ++d) m->t[i].ne[d] = (int64_t)rd64(&c);
    m->t[i].type = (int)rd32(&c);
    off[i] = rd64(&c);
  }
  const size_t data0 = ((size_t)(c.p - m->file) + (size_t)align - 1) / (size_t)align * (size_t)align;
  for (uint64_t i = 0; i < nt; ++i) m->t[i].data = m->file + data0 + off[i];
  free(off);
  m->tok = find_t(m, "token_embd.weight");
  m->out = find_t(m, "output.weight");
  if (!m->out) m->out = m->tok;
  m->onorm = find_t(m, "output_norm.weight");
  if (!m->tok || !m->onorm) {
    orc_model_close(m);
    return NULL;
  }
  m->n_vocab = (int)t_rows(m->out);
  static const char* names[11] = {"attn_norm", "ffn_norm", "attn_q_norm", "attn_k_norm", "attn_q", "attn_k",
                                  "attn_v",    "attn_output", "ffn_gate", "ffn_up", "ffn_down"};
  m->L = (const orc_tensor**)calloc((size_t)m->n_layer * 11, sizeof(orc_tensor*));
  for (int il = 0; il < m->n_layer; ++il) {
    for (int j = 0; j < 11; ++j) {
      char nm[96];
      snprintf(nm, sizeof nm, "blk.%d.%s.weight", il, names[j]);
      m->L[il * 11 + j] = find_t(m, nm);
      if (!m->L[il * 11 + j]) {
        orc_model_close(m);
        return NULL;
      }
    }
  }
  m->n_ctx = n_ctx;
  m->n_seq = n_seq;
  const size_t rows = (size_t)m->n_layer * m->n_head_kv * (size_t)n_seq * n_ctx;
  m->kc = (int8_t*)calloc(rows, (size_t)m->head_dim);
  m->vc = (int8_t*)calloc(rows, (size_t)m->head_dim);
  m->ksc = (float*)calloc(rows, 4);
  m->vsc = (float*)calloc(rows, 4);
  m->inv_freq = (float*)malloc(sizeof(float) * (size_t)(m->head_dim / 2));
  for (int i = 0; i < m->head_dim / 2; ++i)
    m->inv_freq[i] = powf(m->rope_base, -2.0f * (float)i / (float)m->head_dim);
  return m;
}

/* n_layer n_embd n_ff n_head n_head_kv head_dim n_vocab n_ctx n_seq */
void orc_model_cfg(const orc_model* m, int* out) {
  const int v[9] = {m->n_layer, m->n_embd, m->n_ff, m->n_head, m->n_head_kv, m->head_dim, m->n_vocab, m->n_ctx, m->n_seq};
  memcpy(out, v, sizeof v);
}

static size_t kv_index(const orc_model* m, int il, int h, int64_t row) {
  return ((size_t)il * m->n_head_kv + (size_t)h) * ((size_t)m->n_seq * m->n_ctx) + (size_t)row;
}

static void matmul_w(const orc_tensor* w, const float* x, int n, float* y) {
  orc_matmul(w->type, w->data, t_rows(w), w->ne[0], x, n, y);
}

/* Model::forward(const BatchToken*, n, logits) + Model::run (model.cpp:280-430). Returns 0, or -1 on a batch
 * malkin rejects (same checks). */
int orc_model_forward(orc_model* m, int n, const int32_t* id, const int32_t* seq, const int32_t* pos,
                      const int32_t* want, const int32_t* kvp, const int32_t* parent, float* logits) {
  const int E = m->n_embd, D = m->head_dim, H = m->n_head, KV = m->n_head_kv, F = m->n_ff, G = H / KV;
  int *kv_at = (int*)malloc(sizeof(int) * (size_t)n), *kv_base = (int*)malloc(sizeof(int) * (size_t)n),
      *nkeys = (int*)malloc(sizeof(int) * (size_t)n), *aoff = (int*)malloc(sizeof(int) * (size_t)(n + 1)),
      *out = (int*)malloc(sizeof(int) * (size_t)n);
  int* anc = (int*)malloc(sizeof(int) * (size_t)n * (size_t)(n + 1));
  int na = 0, m_out = 0, rc = 0;
  for (int t = 0; t < n; ++t) {
    const int kv = parent[t] < 0 ? pos[t] : kvp[t];
    if (seq[t] < 0 || seq[t] >= m->n_seq || pos[t] < 0 || pos[t] >= m->n_ctx || kv < 0 || kv >= m->n_ctx) rc = -1;
    if (parent[t] >= t || (parent[t] >= 0 && seq[parent[t]] != seq[t])) rc = -1;
    if (id[t] < 0 || id[t] >= t_rows(m->tok)) rc = -1;
    if (rc) break;
    kv_base[t] = seq[t] * m->n_ctx;
    kv_at[t] = kv_base[t] + kv;
    if (want[t]) out[m_out++] = t;
  }
  if (rc) {
    free(kv_at), free(kv_base), free(nkeys), free(aoff), free(out), free(anc);
    return -1;
  }
  for (int t = 0; t < n; ++t) {
    aoff[t] = na;
    if (parent[t] < 0) {
      nkeys[t] = pos[t] + 1;
    } else {
      nkeys[t] = nkeys[parent[t]];
      for (int i = aoff[parent[t]]; i < aoff[parent[t] + 1]; ++i) anc[na++] = anc[i];
      anc[na++] = kv_at[t] - kv_base[t];
    }
    aoff[t + 1] = na;
  }
  const size_t sn = (size_t)n;
  float* x = (float*)malloc(sizeof(float) * sn * E);
  float* h = (float*)malloc(sizeof(float) * sn * (E > F ? E : F));
  float* q = (float*)malloc(sizeof(float) * sn * H * D);
  float* k = (float*)malloc(sizeof(float) * sn * KV * D);
  float* v = (float*)malloc(sizeof(float) * sn * KV * D);
  float* att = (float*)malloc(sizeof(float) * sn * H * D);
  float* gate = (float*)malloc(sizeof(float) * sn * F);
  float* up = (float*)malloc(sizeof(float) * sn * F);
  float* cs = (float*)malloc(sizeof(float) * sn * D);
  const size_t erb = orc_row_bytes(m->tok->type, E);
  for (int t = 0; t < n; ++t) {
    orc_dequantize_row(m->tok->type, m->tok->data + (size_t)id[t] * erb, x + (size_t)t * E, E);
    for (int i = 0; i < D / 2; ++i) {
      const float a = (float)pos[t] * m->inv_freq[i];
      cs[(size_t)t * D + i] = cosf(a);
      cs[(size_t)t * D + D / 2 + i] = sinf(a);
    }
  }
  const float scale = 1.0f / sqrtf((float)D);
  for (int il = 0; il < m->n_layer; ++il) {
    const orc_tensor** L = m->L + il * 11;
    for (int t = 0; t < n; ++t) rmsnorm(h + (size_t)t * E, x + (size_t)t * E, (const float*)L[0]->data, E, m->rms_eps);
    matmul_w(L[4], h, n, q);
    matmul_w(L[5], h, n, k);
    matmul_w(L[6], h, n, v);
    for (int t = 0; t < n; ++t) {
      const float* c0 = cs + (size_t)t * D;
      for (int hh = 0; hh < H + KV; ++hh) {
        float* vv = hh < H ? q + ((size_t)t * H + hh) * D : k + ((size_t)t * KV + (hh - H)) * D;
        rmsnorm(vv, vv, (const float*)(hh < H ? L[2] : L[3])->data, D, m->rms_eps);
        /* RoPE as g++ -O2 -march=x86-64-v4 compiles model.cpp's rope (FMA contraction is on for C++):
         * x0 * cos - x1 * sin -> fma(x0, cos, -(x1 * sin)); x0 * sin + x1 * cos -> fma(x0, sin, x1 * cos) */
        for (int i = 0; i < D / 2; ++i) {
          const float x0 = vv[i], x1 = vv[i + D / 2];
          vv[i] = fmaf(x0, c0[i], -(x1 * c0[D / 2 + i]));
          vv[i + D / 2] = fmaf(x0, c0[D / 2 + i], x1 * c0[i]);
        }
      }
      for (int hh = 0; hh < KV; ++hh) {
        const size_t ki = kv_index(m, il, hh, kv_at[t]);
        m->ksc[ki] = orc_quantize_i8(k + ((size_t)t * KV + hh) * D, D, m->kc + ki * D);
        m->vsc[ki] = orc_quantize_i8(v + ((size_t)t * KV + hh) * D, D, m->vc + ki * D);
      }
    }
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
    for (int t = 0; t < n; ++t) {
      for (int g = 0; g < KV; ++g) {
        const size_t k0 = kv_index(m, il, g, kv_base[t]);
        orc_attend(q + ((size_t)t * H + (size_t)g * G) * D, G, D, m->kc + k0 * D, m->vc + k0 * D, m->ksc + k0,
                   m->vsc + k0, D, nkeys[t], anc + aoff[t], aoff[t + 1] - aoff[t], scale,
                   att + ((size_t)t * H + (size_t)g * G) * D);
      }
    }
    matmul_w(L[7], att, n, h);
    for (size_t i = 0; i < sn * E; ++i) x[i] += h[i];
    for (int t = 0; t < n; ++t) rmsnorm(h + (size_t)t * E, x + (size_t)t * E, (const float*)L[1]->data, E, m->rms_eps);
    matmul_w(L[8], h, n, gate);
    matmul_w(L[9], h, n, up);
    orc_silu_mul((int64_t)n * F, gate, up);
    matmul_w(L[10], gate, n, h);
    for (size_t i = 0; i < sn * E; ++i) x[i] += h[i];
  }
  if (m_out > 0) {
    for (int i = 0; i < m_out; ++i)
      rmsnorm(h + (size_t)i * E, x + (size_t)out[i] * E, (const float*)m->onorm->data, E, m->rms_eps);
    matmul_w(m->out, h, m_out, logits);
  }
  free(x), free(h), free(q), free(k), free(v), free(att), free(gate), free(up), free(cs);
  free(kv_at), free(kv_base), free(nkeys), free(aoff), free(out), free(anc);
  return 0;
}

/* Model::move_kv (model.cpp:432-440) */
void orc_model_move_kv(orc_model* m, int from, int to, int seq) {
  if (from == to) return;
  const int64_t b = (int64_t)seq * m->n_ctx;
  for (int il = 0; il < m->n_layer; ++il) {
    for (int h = 0; h < m->n_head_kv; ++h) {
      const size_t f = kv_index(m, il, h, b + from), t = kv_index(m, il, h, b + to);
      memcpy(m->kc + t * m->head_dim, m->kc + f * m->head_dim, (size_t)m->head_dim);
      memcpy(m->vc + t * m->head_dim, m->vc + f * m->head_dim, (size_t)m->head_dim);
      m->ksc[t] = m->ksc[f];
      m->vsc[t] = m->vsc[f];
    }
  }
}

/* ---------------- sampler + accept (sampler.cpp:22-97, engine.cpp:441-507) ---------------- */

typedef struct {
  float temperature, top_p, min_p;
  int top_k;
} orc_sampling;

/* Sampler::distribution without penalties: greedy -> [(1, argmax)]; else top-k (value desc, index asc on ties),
 * exp((l - max) / T) in float, min-p then nucleus in double, normalised. Returns the entry count. */
int orc_distribution(const float* logits, int V, orc_sampling s, float* p, int32_t* ids) {
  if (s.temperature <= 0.0f) {
    int best = 0;
    for (int i = 1; i < V; ++i)
      if (logits[i] > logits[best]) best = i;
    p[0] = 1.0f;
    ids[0] = best;
    return 1;
  }
  const int k = s.top_k > 0 && s.top_k < V ? s.top_k : V;
  float* cv = (float*)malloc(sizeof(float) * (size_t)k);
  int* ci = (int*)malloc(sizeof(int) * (size_t)k);
  int nc = 0;
  for (int i = 0; i < V; ++i) { /* insertion into a sorted top-k list */
    const float v = logits[i];
    if (nc == k && !(v > cv[k - 1])) continue;
    int j = nc < k ? nc++ : k - 1;
    while (j > 0 && v > cv[j - 1]) {
      cv[j] = cv[j - 1];
      ci[j] = ci[j - 1];
      --j;
    }
    cv[j] = v;
    ci[j] = i;
  }
  float* e = (float*)malloc(sizeof(float) * (size_t)k);
  const float mx = cv[0];
  double sum = 0.0;
  for (int j = 0; j < k; ++j) {
    e[j] = expf((cv[j] - mx) / s.temperature);
    sum += e[j];
  }
  const double floor = (double)s.min_p * e[0];
  double kept = 0.0;
  int n = 0;
  for (; n < k; ++n) {
    if (n > 0 && e[n] < floor) break;
    kept += e[n];
    if (kept >= s.top_p * sum) {
      ++n;
      break;
    }
  }
  if (n < 1) n = 1;
  double total = 0.0;
  for (int j = 0; j < n; ++j) total += e[j];
  for (int j = 0; j < n; ++j) {
    p[j] = (float)(e[j] / total);
    ids[j] = ci[j];
  }
  free(cv), free(ci), free(e);
  return n;
}

static float prob_of(const float* p, const int32_t* id, int n, int d) {
  for (int j = 0; j < n; ++j)
    if (id[j] == d) return p[j];
  return 0.0f;
}

/* Sampler::draw (sampler.cpp:64-72) */
static int draw(const float* p, const int32_t* id, int n, const double* U, int* u) {
  if (n == 1) return id[0];
  double r = U[(*u)++];
  for (int j = 0; j < n; ++j) {
    r -= p[j];
    if (r <= 0) return id[j];
  }
  return id[n - 1];
}

/* Engine::accept_greedy (engine.cpp:441-479) on the logits rows of one slot (row t = tree node t). Moves the KV of
 * accepted nodes when m != NULL. Returns the accepted count; *next, *last_node. */
int orc_accept_greedy(orc_model* m, const float* logits, int V, int kk, const int32_t* chain, const int32_t* alt,
                      int seq, int cache_len, int32_t* acc_ids, int32_t* next, int32_t* last_node) {
  const int P = cache_len;
  int size = P + 1, cur = 0, n = 0, bonus = 0;
  float pp;
  int32_t a;
  orc_sampling g = {0.0f, 1.0f, 0.0f, 0};
  for (int i = 0; i < kk; ++i) {
    orc_distribution(logits + (size_t)cur * V, V, g, &pp, &a);
    int slot = -1;
    if (a == chain[i])
      slot = 1 + 2 * i;
    else if (a == alt[i])
      slot = 2 + 2 * i;
    if (slot < 0) {
      *next = a;
      bonus = 1;
      break;
    }
    if (m) orc_model_move_kv(m, P + slot, size, seq);
    ++size;
    acc_ids[n++] = a;
    cur = slot;
    if (slot == 2 + 2 * i) break;
  }
  if (!bonus) {
    orc_distribution(logits + (size_t)cur * V, V, g, &pp, &a);
    *next = a;
  }
  *last_node = cur;
  return n;
}

/* Engine::accept_sampled + Sampler::verify (engine.cpp:482-507, sampler.cpp:80-97) with the uniform stream U.
 * Rows 0..kk of logits: [next, d0, ...]. Returns the accepted count; *next, *u_used. */
int orc_accept_sampled(const float* logits, int V, orc_sampling s, int kk, const int32_t* chain, const float* q_p,
                       const int32_t* q_id, const int32_t* q_n, const double* U, int32_t* acc_ids, int32_t* next,
                       int32_t* u_used) {
  float* p = (float*)malloc(sizeof(float) * (size_t)(s.top_k > 0 ? s.top_k : V));
  int32_t* pid = (int32_t*)malloc(sizeof(int32_t) * (size_t)(s.top_k > 0 ? s.top_k : V));
  float* rp = (float*)malloc(sizeof(float) * (size_t)(s.top_k > 0 ? s.top_k : V));
  int32_t* rid = (int32_t*)malloc(sizeof(int32_t) * (size_t)(s.top_k > 0 ? s.top_k : V));
  int u = 0, i = 0, n = 0, qo = 0;
  for (; i < kk; ++i) {
    const int np = orc_distribution(logits + (size_t)i * V, V, s, p, pid);
    const int d = chain[i];
    const float pd = prob_of(p, pid, np, d), qd = prob_of(q_p + qo, q_id + qo, q_n[i], d);
    const double uu = U[u++];
    if (qd > 0.0f && uu * qd < pd) {
      acc_ids[n++] = d;
      qo += q_n[i];
      continue;
    }
    int nr = 0;
    double total = 0.0;
    for (int j = 0; j < np; ++j) {
      const float r = p[j] - prob_of(q_p + qo, q_id + qo, q_n[i], pid[j]);
      if (r > 0.0f) {
        rp[nr] = r;
        rid[nr++] = pid[j];
        total += r;
      }
    }
    if (nr == 0) {
      *next = draw(p, pid, np, U, &u);
    } else {
      for (int j = 0; j < nr; ++j) rp[j] = (float)(rp[j] / total);
      *next = draw(rp, rid, nr, U, &u);
    }
    break;
  }
  if (i == kk) {
    const int np = orc_distribution(logits + (size_t)kk * V, V, s, p, pid);
    *next = draw(p, pid, np, U, &u);
  }
  *u_used = u;
  free(p), free(pid), free(rp), free(rid);
  return n;
}
