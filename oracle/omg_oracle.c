/*
 * omg_oracle.c — TEST INFRASTRUCTURE ONLY (see omg_oracle.h).
 *
 * Plain C restatement of the reference's CPU code for the omg-wgpu forward
 * pass. Built with -ffp-contract=off so a*b+c rounds twice, as Rust does.
 * The one liberty taken: dot products accumulate in 8 interleaved partial
 * sums (added in a fixed order) instead of one running sum, so the compiler
 * can vectorise them; that reassociates f32 additions only.
 */
#include "omg_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ---- f16 ----------------------------------------------------------------- */

uint16_t oracle_f32_to_f16(float v) {
  uint32_t x;
  memcpy(&x, &v, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t exp = (x >> 23) & 0xffu;
  const uint32_t man = x & 0x7fffffu;
  if (exp == 0xffu) {
    if (man) return (uint16_t)(sign | 0x7e00u | (man >> 13));
    return (uint16_t)(sign | 0x7c00u);
  }
  const int e = (int)exp - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7c00u);
  if (e <= 0) {
    /* Subnormal half: m * 2^-24 with m = (1.man) * 2^(exp - 126). */
    const int shift = 126 - (int)exp;
    if (shift > 25) return (uint16_t)sign;
    const uint64_t full = (uint64_t)(man | 0x800000u);
    uint64_t m = full >> shift;
    const uint64_t rem = full & ((1ull << shift) - 1ull);
    const uint64_t half = 1ull << (shift - 1);
    if (rem > half || (rem == half && (m & 1ull))) m++;
    return (uint16_t)(sign | (uint32_t)m);
  }
  uint32_t h = sign | ((uint32_t)e << 10) | (man >> 13);
  const uint32_t rem = man & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
  return (uint16_t)h;
}

float oracle_f16_to_f32(uint16_t h) {
  const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  uint32_t x;
  if (exp == 0x1fu) {
    x = sign | 0x7f800000u | (man << 13);
  } else if (exp == 0) {
    if (man == 0) {
      x = sign;
    } else {
      int e = -1;
      do {
        e++;
        man <<= 1;
      } while (!(man & 0x400u));
      man &= 0x3ffu;
      x = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else {
    x = sign | ((exp - 15 + 127) << 23) | (man << 13);
  }
  float v;
  memcpy(&v, &x, 4);
  return v;
}

void oracle_f32_to_f16_n(const float* in, size_t n, uint16_t* out) {
  for (size_t i = 0; i < n; ++i) out[i] = oracle_f32_to_f16(in[i]);
}

void oracle_f16_to_f32_n(const uint16_t* in, size_t n, float* out) {
  for (size_t i = 0; i < n; ++i) out[i] = oracle_f16_to_f32(in[i]);
}

static float round_f16(float v) { return oracle_f16_to_f32(oracle_f32_to_f16(v)); }

/* ---- xorshift (tests/reference.rs:17-26) ---------------------------------- */

void oracle_rng_values(uint64_t* state, float* out, size_t n, float scale) {
  uint64_t s = *state;
  for (size_t i = 0; i < n; ++i) {
    s ^= s << 13;
    s ^= s >> 7;
    s ^= s << 17;
    const float u = ((float)(s >> 40) / (float)(1ull << 24)) * 2.0f - 1.0f;
    out[i] = u * scale;
  }
  *state = s;
}

/* ---- synthetic weights ------------------------------------------------------
 * The benchmark's and the large-shape tests' random models: a normal draw per
 * element from xorshift64 (seeded by FNV-1a(name) ^ seed; 53-bit uniforms in
 * (0, 1)) through the Box-Muller transform in double precision, rounded to
 * f32. The product library generates its models with the same definition;
 * this copy lets CPU-only runs build the same weights without loading it. */
void oracle_synth_normal(uint64_t seed, const char* name, float mean, float stddev, float* out,
                         size_t n) {
  uint64_t s = 0xcbf29ce484222325ull;
  for (const char* p = name ? name : ""; *p; ++p) {
    s ^= (uint8_t)*p;
    s *= 0x00000100000001b3ull;
  }
  s ^= seed;
  if (s == 0) s = 0x9e3779b97f4a7c15ull;
  const double two_pi = 6.283185307179586;
  for (size_t i = 0; i < n; i += 2) {
    double u[2];
    for (int j = 0; j < 2; ++j) {
      s ^= s << 13;
      s ^= s >> 7;
      s ^= s << 17;
      u[j] = ((double)(s >> 11) + 0.5) * (1.0 / 9007199254740992.0);
    }
    const double r = sqrt(-2.0 * log(u[0]));
    out[i] = (float)(mean + stddev * r * cos(two_pi * u[1]));
    if (i + 1 < n) out[i + 1] = (float)(mean + stddev * r * sin(two_pi * u[1]));
  }
}

/* ---- quantizers (model.rs:409-466) --------------------------------------- */

static void put_f16(uint8_t* p, float v) {
  const uint16_t h = oracle_f32_to_f16(v);
  p[0] = (uint8_t)(h & 0xff);
  p[1] = (uint8_t)(h >> 8);
}

static float get_f16(const uint8_t* p) {
  return oracle_f16_to_f32((uint16_t)(p[0] | ((uint16_t)p[1] << 8)));
}

int oracle_quantize_q8(const float* v, size_t n, uint8_t* codes, uint8_t* scales) {
  if (n % 32) return -1;
  for (size_t b = 0; b < n / 32; ++b) {
    const float* blk = v + 32 * b;
    float amax = 0.0f;
    for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(blk[j]));
    const float d = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    put_f16(scales + 2 * b, d);
    for (int j = 0; j < 32; ++j) {
      float q = roundf(blk[j] * id);
      if (q < -127.0f) q = -127.0f;
      if (q > 127.0f) q = 127.0f;
      codes[32 * b + j] = (uint8_t)(int8_t)q;
    }
  }
  return 0;
}

static int clamp_trunc(float x) {
  /* Rust `as i32` (truncation, saturating), then clamp(0, 15). */
  int q;
  if (!(x == x)) q = 0;
  else if (x >= 2147483647.0f) q = 2147483647;
  else if (x <= -2147483648.0f) q = (-2147483647 - 1);
  else q = (int)x;
  if (q < 0) q = 0;
  if (q > 15) q = 15;
  return q;
}

int oracle_quantize_q4(const float* v, size_t n, uint8_t* codes, uint8_t* scales) {
  if (n % 32) return -1;
  for (size_t b = 0; b < n / 32; ++b) {
    const float* blk = v + 32 * b;
    float max = 0.0f, amax = 0.0f;
    for (int j = 0; j < 32; ++j) {
      if (fabsf(blk[j]) > amax) {
        amax = fabsf(blk[j]);
        max = blk[j];
      }
    }
    const float d = max / -8.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    put_f16(scales + 2 * b, d);
    for (int j = 0; j < 16; ++j) {
      const int lo = clamp_trunc(blk[j] * id + 8.5f);
      const int hi = clamp_trunc(blk[j + 16] * id + 8.5f);
      codes[16 * b + j] = (uint8_t)(lo | (hi << 4));
    }
  }
  return 0;
}

int oracle_dequant(int dtype, const uint8_t* codes, const uint8_t* scales, size_t n, float* out) {
  for (size_t i = 0; i < n; ++i) {
    if (dtype == 0) {
      out[i] = get_f16(codes + 2 * i);
    } else if (dtype == 1) {
      const float d = get_f16(scales + 2 * (i / 32));
      out[i] = (float)(int8_t)codes[i] * d;
    } else if (dtype == 2) {
      const size_t b = i / 32, j = i % 32;
      const float d = get_f16(scales + 2 * b);
      const uint8_t byte = codes[b * 16 + j % 16];
      const uint8_t q = j < 16 ? (byte & 0xf) : (byte >> 4);
      out[i] = ((float)q - 8.0f) * d;
    } else {
      return -1;
    }
  }
  return 0;
}

/* ---- forward helpers (tests/reference.rs:141-172) ------------------------- */

static float dot8(const float* a, const float* b, int n) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int i = 0;
  for (; i + 8 <= n; i += 8)
    for (int j = 0; j < 8; ++j) acc[j] += a[i + j] * b[i + j];
  float s = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
  for (; i < n; ++i) s += a[i] * b[i];
  return s;
}

/* reference.rs:141-148 */
static void rmsnorm(const float* x, int n, const float* w, float eps, float offset, float* out) {
  float ms = 0.0f;
  for (int i = 0; i < n; ++i) ms += x[i] * x[i];
  ms /= (float)n;
  const float inv = 1.0f / sqrtf(ms + eps);
  for (int i = 0; i < n; ++i) out[i] = x[i] * inv * (w ? offset + w[i] : 1.0f);
}

/* dot8 of four rows of X against two rows of W at once: eight independent
 * 8-lane partial sums, each lane accumulating exactly as dot8 does (mul, then
 * add, in k order) and reduced by the same tree, so every output has dot8's
 * bits; the blocking only keeps more independent sums in flight. */
typedef float v8f __attribute__((vector_size(32)));
static inline v8f ld8(const float* p) {
  v8f v;
  memcpy(&v, p, sizeof v);
  return v;
}
static inline float tree8(v8f a) {
  return ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
}
/* Partial dot8 sums of a 4 x 2 register tile over k in [k0, k1) (k1 - k0 a
 * multiple of 8), carried in `acc` between calls. */
static inline void dot8_4x2_part(const float* x, size_t ldx, const float* w, size_t ldw, int k0,
                                 int k1, v8f acc[4][2]) {
  v8f a00 = acc[0][0], a01 = acc[0][1], a10 = acc[1][0], a11 = acc[1][1];
  v8f a20 = acc[2][0], a21 = acc[2][1], a30 = acc[3][0], a31 = acc[3][1];
  for (int i = k0; i < k1; i += 8) {
    const v8f b0 = ld8(w + i), b1 = ld8(w + ldw + i);
    v8f a = ld8(x + i);
    a00 += a * b0;
    a01 += a * b1;
    a = ld8(x + ldx + i);
    a10 += a * b0;
    a11 += a * b1;
    a = ld8(x + 2 * ldx + i);
    a20 += a * b0;
    a21 += a * b1;
    a = ld8(x + 3 * ldx + i);
    a30 += a * b0;
    a31 += a * b1;
  }
  acc[0][0] = a00, acc[0][1] = a01, acc[1][0] = a10, acc[1][1] = a11;
  acc[2][0] = a20, acc[2][1] = a21, acc[3][0] = a30, acc[3][1] = a31;
}

/* reference.rs:151-157 for every row of X [t, k]: Y [t, n] = X W^T. Blocks of
 * 32 rows x 32 outputs, walked in K chunks of 256 (a chunk of the block's
 * operands stays in the core's L1) with 4 x 2 register tiles whose partial
 * sums carry across chunks; every output keeps dot8's exact arithmetic (each
 * of its 8 lanes accumulates mul-then-add in k order, reduced by dot8's
 * tree, then the tail). dot8 itself for the ragged rows and outputs. */
static void linear_rows(const float* x, int t, int k, const float* w, int n, int mode, float* y,
                        int threads) {
  const float* xs = x;
  const float* ws = w;
  float* xr = NULL;
  float* wr = NULL;
  if (mode == ORACLE_KERNEL) {
    xr = (float*)malloc(sizeof(float) * (size_t)t * k);
    wr = (float*)malloc(sizeof(float) * (size_t)n * k);
#pragma omp parallel for schedule(static) num_threads(threads)
    for (size_t i = 0; i < (size_t)t * k; ++i) xr[i] = round_f16(x[i]);
#pragma omp parallel for schedule(static) num_threads(threads)
    for (size_t i = 0; i < (size_t)n * k; ++i) wr[i] = round_f16(w[i]);
    xs = xr;
    ws = wr;
  }
  enum { BT = 32, BN = 32, KC = 256 };
  const int tb = (t + BT - 1) / BT, nb = (n + BN - 1) / BN;
  const int k8 = k / 8 * 8;
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads)
  for (int blk = 0; blk < tb * nb; ++blk) {
    const int i0 = (blk % tb) * BT, r0 = (blk / tb) * BN;
    const int i1 = i0 + BT < t ? i0 + BT : t, r1 = r0 + BN < n ? r0 + BN : n;
    const int iq = i0 + (i1 - i0) / 4 * 4, rp = r0 + (r1 - r0) / 2 * 2;
    v8f acc[BT / 4][BN / 2][4][2];
    memset(acc, 0, sizeof acc);
    for (int kc = 0; kc < k8; kc += KC) {
      const int ke = kc + KC < k8 ? kc + KC : k8;
      for (int r = r0; r < rp; r += 2)
        for (int i = i0; i < iq; i += 4)
          dot8_4x2_part(xs + (size_t)i * k, (size_t)k, ws + (size_t)r * k, (size_t)k, kc, ke,
                        acc[(i - i0) / 4][(r - r0) / 2]);
    }
    for (int r = r0; r < rp; r += 2)
      for (int i = i0; i < iq; i += 4)
        for (int a = 0; a < 4; ++a)
          for (int c = 0; c < 2; ++c) {
            float s = tree8(acc[(i - i0) / 4][(r - r0) / 2][a][c]);
            for (int j = k8; j < k; ++j)
              s += xs[(size_t)(i + a) * k + j] * ws[(size_t)(r + c) * k + j];
            y[(size_t)(i + a) * n + r + c] = s;
          }
    for (int r = r0; r < r1; ++r)
      for (int i = (r < rp ? iq : i0); i < i1; ++i)
        y[(size_t)i * n + r] = dot8(xs + (size_t)i * k, ws + (size_t)r * k, k);
  }
  free(xr);
  free(wr);
}

/* reference.rs:159-168 */
static void rope(float* v, int len, int pos, float theta, int rope_dims) {
  const int half = len / 2;
  for (int i = 0; i < rope_dims / 2; ++i) {
    const float ang = (float)pos * powf(theta, -(float)i / (float)half);
    const float s = sinf(ang), c = cosf(ang);
    const float a = v[i], b = v[i + half];
    v[i] = a * c - b * s;
    v[i + half] = b * c + a * s;
  }
}

/* reference.rs:170-172 */
static float gelu(float x) {
  return 0.5f * x * (1.0f + tanhf(0.7978845608f * (x + 0.044715f * x * x * x)));
}

int oracle_visible(int32_t qp, int32_t qs, int32_t kp, int32_t ks, int window) {
  const int same_group = ((ks ^ qs) >> 12) == 0;
  return same_group && ((ks & 0xfff) == 0 || ks == qs) && kp <= qp &&
         (window == 0 || (uint32_t)(qp - kp) < (uint32_t)window);
}

/* ---- the forward (tests/reference.rs:175-349) ----------------------------- */

typedef struct {
  const float *attn_norm, *qkv, *q_norm, *k_norm, *o, *post_attn_norm, *ffn_norm, *gate, *up,
      *down, *post_ffn_norm, *pl_gate, *pl_proj, *pl_norm;
  float out_scale;
} layer_w;

int oracle_forward_layers(const oracle_config* cfg, const float* const* tensors,
                          size_t n_tensors, const uint32_t* ids, const int32_t* pos,
                          const int32_t* seq, size_t t_, int mode, int threads, float* hidden,
                          float* per_layer) {
  const int d = cfg->d, L = cfg->layers, heads = cfg->heads, kvh = cfg->kv_heads;
  const int pl = cfg->per_layer_dim;
  const int t = (int)t_;
  if (threads <= 0) {
#ifdef _OPENMP
    threads = omp_get_max_threads();
#else
    threads = 1;
#endif
  }
  /* Catalogue order of Config::tensors (model.rs:277-314). */
  size_t ti = 0;
#define NEXT() (ti < n_tensors ? tensors[ti++] : NULL)
  const float* embed = NEXT();
  const float* final_norm = NEXT();
  const float* pl_model_proj = NULL;
  const float* pl_proj_norm = NULL;
  if (pl > 0) {
    pl_model_proj = NEXT();
    pl_proj_norm = NEXT();
  }
  layer_w* lw = (layer_w*)calloc((size_t)L, sizeof(layer_w));
  for (int l = 0; l < L; ++l) {
    const int has_kv = cfg->kv_source[l] == l;
    lw[l].attn_norm = NEXT();
    lw[l].qkv = NEXT();
    lw[l].q_norm = NEXT();
    lw[l].k_norm = has_kv ? NEXT() : NULL;
    lw[l].o = NEXT();
    lw[l].post_attn_norm = NEXT();
    lw[l].ffn_norm = NEXT();
    lw[l].gate = NEXT();
    lw[l].up = NEXT();
    lw[l].down = NEXT();
    lw[l].post_ffn_norm = NEXT();
    lw[l].out_scale = 1.0f;
    if (pl > 0) {
      lw[l].pl_gate = NEXT();
      lw[l].pl_proj = NEXT();
      lw[l].pl_norm = NEXT();
      const float* os = NEXT();
      lw[l].out_scale = os ? os[0] : 1.0f;
    }
  }
  const float* pl_table = pl > 0 ? NEXT() : NULL;
#undef NEXT
  if (ti != n_tensors || !embed || !final_norm) {
    free(lw);
    return -1;
  }
  for (int i = 0; i < t; ++i)
    if ((int)ids[i] >= cfg->vocab) {
      free(lw);
      return -2;
    }

  int max_hd = 0, max_ff = 0, max_qkv = 0;
  for (int l = 0; l < L; ++l) {
    if (cfg->head_dim[l] > max_hd) max_hd = cfg->head_dim[l];
    if (cfg->ff[l] > max_ff) max_ff = cfg->ff[l];
    const int w = (cfg->kv_source[l] == l ? heads + 2 * kvh : heads) * cfg->head_dim[l];
    if (w > max_qkv) max_qkv = w;
  }
  const size_t T = (size_t)t;
  float* x = (float*)malloc(sizeof(float) * T * d);
  float* h = (float*)malloc(sizeof(float) * T * d);
  float* qkv = (float*)malloc(sizeof(float) * T * max_qkv);
  float* q = (float*)malloc(sizeof(float) * T * heads * max_hd);
  float* attn = (float*)malloc(sizeof(float) * T * heads * max_hd);
  float* a = (float*)malloc(sizeof(float) * T * d);
  float* gt = (float*)malloc(sizeof(float) * T * max_ff);
  float* u = (float*)malloc(sizeof(float) * T * max_ff);
  float* big = (float*)malloc(sizeof(float) * T * (max_ff > d ? max_ff : d));
  float** kv_k = (float**)calloc((size_t)L, sizeof(float*));
  float** kv_v = (float**)calloc((size_t)L, sizeof(float*));
  float* pli = pl > 0 ? (float*)malloc(sizeof(float) * T * pl * L) : NULL;

  /* Embedding times sqrt(d) (reference.rs:183-191). */
  const float sd = sqrtf((float)d);
  for (int i = 0; i < t; ++i)
    for (int k = 0; k < d; ++k) x[(size_t)i * d + k] = embed[(size_t)ids[i] * d + k] * sd;

  /* Per-layer inputs (reference.rs:193-222). */
  if (pl > 0) {
    float* p = (float*)malloc(sizeof(float) * T * pl * L);
    linear_rows(x, t, d, pl_model_proj, pl * L, mode, p, threads);
    float* sl = (float*)malloc(sizeof(float) * pl);
    float* nn = (float*)malloc(sizeof(float) * pl);
    for (int i = 0; i < t; ++i)
      for (int l = 0; l < L; ++l) {
        for (int j = 0; j < pl; ++j) sl[j] = p[(size_t)i * pl * L + l * pl + j] / sd;
        rmsnorm(sl, pl, pl_proj_norm, cfg->eps, cfg->norm_offset, nn);
        for (int j = 0; j < pl; ++j) {
          const float e =
              pl_table[(size_t)ids[i] * pl * L + l * pl + j] * sqrtf((float)pl);
          pli[(size_t)i * pl * L + l * pl + j] = (nn[j] + e) / sqrtf(2.0f);
        }
      }
    free(p);
    free(sl);
    free(nn);
  }

  for (int li = 0; li < L; ++li) {
    const layer_w* W = &lw[li];
    const int hd = cfg->head_dim[li];
    const int sliding = cfg->sliding[li];
    const float theta = sliding ? cfg->theta_local : cfg->theta_global;
    const int has_kv = cfg->kv_source[li] == li;
    const int hpg = heads / kvh;
    const int qkv_w = (has_kv ? heads + 2 * kvh : heads) * hd;

    for (int i = 0; i < t; ++i)
      rmsnorm(x + (size_t)i * d, d, W->attn_norm, cfg->eps, cfg->norm_offset, h + (size_t)i * d);
    linear_rows(h, t, d, W->qkv, qkv_w, mode, qkv, threads);
    if (has_kv) {
      kv_k[li] = (float*)malloc(sizeof(float) * T * kvh * hd);
      kv_v[li] = (float*)malloc(sizeof(float) * T * kvh * hd);
    }
#pragma omp parallel for schedule(static) num_threads(threads)
    for (int i = 0; i < t; ++i) {
      const float* row = qkv + (size_t)i * qkv_w;
      float tmp[1024];
      for (int hh = 0; hh < heads; ++hh) {
        rmsnorm(row + hh * hd, hd, W->q_norm, cfg->eps, cfg->norm_offset, tmp);
        rope(tmp, hd, pos[i], theta, cfg->rope_dims[li]);
        for (int dd = 0; dd < hd; ++dd)
          q[(size_t)i * heads * hd + hh * hd + dd] = tmp[dd] * cfg->query_scale;
      }
      if (has_kv) {
        for (int gh = 0; gh < kvh; ++gh) {
          rmsnorm(row + (heads + gh) * hd, hd, W->k_norm, cfg->eps, cfg->norm_offset, tmp);
          rope(tmp, hd, pos[i], theta, cfg->rope_dims[li]);
          memcpy(kv_k[li] + (size_t)i * kvh * hd + gh * hd, tmp, sizeof(float) * hd);
          const float* vv = row + (heads + kvh + gh) * hd;
          float* vo = kv_v[li] + (size_t)i * kvh * hd + gh * hd;
          if (cfg->v_norm)
            rmsnorm(vv, hd, NULL, cfg->eps, 0.0f, vo);
          else
            memcpy(vo, vv, sizeof(float) * hd);
        }
      }
    }
    const float* K = kv_k[cfg->kv_source[li]];
    const float* V = kv_v[cfg->kv_source[li]];
    const int window = sliding ? cfg->window : 0;
#pragma omp parallel for schedule(dynamic, 4) num_threads(threads)
    for (int i = 0; i < t; ++i) {
      float* sc = (float*)malloc(sizeof(float) * T);
      int* idx = (int*)malloc(sizeof(int) * T);
      float qh[1024], kj[1024];
      float* out = attn + (size_t)i * heads * hd;
      for (int k = 0; k < heads * hd; ++k) out[k] = 0.0f;
      for (int hh = 0; hh < heads; ++hh) {
        const int gh = hh / hpg;
        for (int dd = 0; dd < hd; ++dd) {
          const float v = q[(size_t)i * heads * hd + hh * hd + dd];
          qh[dd] = mode == ORACLE_KERNEL ? round_f16(v) : v;
        }
        int n = 0;
        for (int j = 0; j < t; ++j) {
          if (!oracle_visible(pos[i], seq[i], pos[j], seq[j], window)) continue;
          const float* kr = K + (size_t)j * kvh * hd + gh * hd;
          if (mode == ORACLE_KERNEL) {
            for (int dd = 0; dd < hd; ++dd) kj[dd] = round_f16(kr[dd]);
            sc[n] = dot8(qh, kj, hd);
          } else {
            sc[n] = dot8(qh, kr, hd);
          }
          idx[n++] = j;
        }
        float m = -3.402823466e38f; /* f32::MIN */
        for (int s = 0; s < n; ++s) m = fmaxf(m, sc[s]);
        float lsum = 0.0f;
        for (int s = 0; s < n; ++s) lsum += expf(sc[s] - m);
        for (int s = 0; s < n; ++s) {
          const float p = expf(sc[s] - m) / lsum;
          const float* vr = V + (size_t)idx[s] * kvh * hd + gh * hd;
          for (int dd = 0; dd < hd; ++dd) {
            const float vv = mode == ORACLE_KERNEL ? round_f16(vr[dd]) : vr[dd];
            out[hh * hd + dd] += p * vv;
          }
        }
      }
      free(sc);
      free(idx);
    }
    /* x += post_attn_norm(attn o^T) (reference.rs:286-296) */
    linear_rows(attn, t, heads * hd, W->o, d, mode, a, threads);
    for (int i = 0; i < t; ++i) {
      float* xi = x + (size_t)i * d;
      rmsnorm(a + (size_t)i * d, d, W->post_attn_norm, cfg->eps, cfg->norm_offset, big);
      for (int dd = 0; dd < d; ++dd) xi[dd] += big[dd];
      rmsnorm(xi, d, W->ffn_norm, cfg->eps, cfg->norm_offset, h + (size_t)i * d);
    }
    /* GeGLU (reference.rs:297-300) */
    const int ff = cfg->ff[li];
    linear_rows(h, t, d, W->gate, ff, mode, gt, threads);
    linear_rows(h, t, d, W->up, ff, mode, u, threads);
    for (size_t k = 0; k < T * ff; ++k) big[k] = gelu(gt[k]) * u[k];
    linear_rows(big, t, ff, W->down, d, mode, a, threads);
    for (int i = 0; i < t; ++i) {
      float* xi = x + (size_t)i * d;
      float tmp[8192];
      rmsnorm(a + (size_t)i * d, d, W->post_ffn_norm, cfg->eps, cfg->norm_offset, tmp);
      for (int dd = 0; dd < d; ++dd) xi[dd] += tmp[dd];
    }
    float scale = 1.0f;
    if (pl > 0) {
      /* reference.rs:310-330 */
      float* gate = (float*)malloc(sizeof(float) * T * pl);
      float* gated = (float*)malloc(sizeof(float) * T * pl);
      linear_rows(x, t, d, W->pl_gate, pl, mode, gate, threads);
      for (int i = 0; i < t; ++i)
        for (int j = 0; j < pl; ++j)
          gated[(size_t)i * pl + j] =
              gelu(gate[(size_t)i * pl + j]) * pli[(size_t)i * pl * L + li * pl + j];
      linear_rows(gated, t, pl, W->pl_proj, d, mode, a, threads);
      for (int i = 0; i < t; ++i) {
        float tmp[8192];
        rmsnorm(a + (size_t)i * d, d, W->pl_norm, cfg->eps, cfg->norm_offset, tmp);
        for (int dd = 0; dd < d; ++dd) x[(size_t)i * d + dd] += tmp[dd];
      }
      scale = W->out_scale;
      free(gate);
      free(gated);
    }
    for (size_t k = 0; k < T * d; ++k) x[k] *= scale;
    /* What a model cut after this layer would return: its final norm of
     * the stream. */
    if (per_layer)
      for (int i = 0; i < t; ++i)
        rmsnorm(x + (size_t)i * d, d, final_norm, cfg->eps, cfg->norm_offset,
                per_layer + ((size_t)li * T + i) * d);
  }
  for (int i = 0; i < t; ++i)
    rmsnorm(x + (size_t)i * d, d, final_norm, cfg->eps, cfg->norm_offset, hidden + (size_t)i * d);

  for (int l = 0; l < L; ++l) {
    free(kv_k[l]);
    free(kv_v[l]);
  }
  free(kv_k);
  free(kv_v);
  free(x);
  free(h);
  free(qkv);
  free(q);
  free(attn);
  free(a);
  free(gt);
  free(u);
  free(big);
  free(pli);
  free(lw);
  return 0;
}

int oracle_forward(const oracle_config* cfg, const float* const* tensors, size_t n_tensors,
                   const uint32_t* ids, const int32_t* pos, const int32_t* seq, size_t t,
                   int mode, int threads, float* hidden) {
  return oracle_forward_layers(cfg, tensors, n_tensors, ids, pos, seq, t, mode, threads, hidden,
                               NULL);
}

/* ---- logits and readout --------------------------------------------------- */

void oracle_logits(const float* hidden, const float* embed, int vocab, int d, float softcap,
                   float* out) {
#pragma omp parallel for schedule(static)
  for (int v = 0; v < vocab; ++v) {
    float z = 0.0f;
    for (int i = 0; i < d; ++i) z += hidden[i] * embed[(size_t)v * d + i];
    out[v] = softcap > 0.0f ? softcap * tanhf(z / softcap) : z;
  }
}

void oracle_softmax(const float* z, size_t n, float temperature, double* out) {
  const double t = (double)(temperature > 1e-6f ? temperature : 1e-6f);
  float m = -INFINITY;
  for (size_t i = 0; i < n; ++i) m = fmaxf(m, z[i]);
  double s = 0.0;
  for (size_t i = 0; i < n; ++i) {
    out[i] = exp(((double)z[i] - (double)m) / t);
    s += out[i];
  }
  for (size_t i = 0; i < n; ++i) out[i] /= s;
}

double oracle_log_sum_exp(const float* z, size_t n) {
  float m = -INFINITY;
  for (size_t i = 0; i < n; ++i) m = fmaxf(m, z[i]);
  double s = 0.0;
  for (size_t i = 0; i < n; ++i) s += exp((double)z[i] - (double)m);
  return (double)m + log(s);
}

/* ---- Laya / ModernBERT encoder (crates/omg-wgpu/src/laya.rs) --------------
 *
 * The reference has no CPU code for this path; this restates the GPU plan
 * of LayaEngine::hidden (laya.rs:1263-1345) kernel by kernel: embed.wgsl,
 * layernorm.wgsl:48-68, rope_bi.wgsl:16-44, attention_bi.wgsl:59-188,
 * matmul_gated.wgsl:114-134 (erf GELU), bias_act.wgsl:26-40, and the host
 * scorer / act head of laya.rs:1442-1493. */

/* layernorm.wgsl:48-68: optional residual update x += a (+ rb), then
 * y = (v - mean) * rsqrt(var + eps) * w (+ b), variance around the mean. */
static void laya_ln_row(float* x, const float* a, const float* rb, const float* w, const float* b,
                        int d, float eps, float* out) {
  if (a) {
    for (int i = 0; i < d; ++i) {
      float e = x[i] + a[i];
      if (rb) e += rb[i];
      x[i] = e;
    }
  }
  float s = 0.0f;
  for (int i = 0; i < d; ++i) s += x[i];
  const float mean = s / (float)d;
  float q = 0.0f;
  for (int i = 0; i < d; ++i) {
    const float c = x[i] - mean;
    q += c * c;
  }
  const float inv = 1.0f / sqrtf(q / (float)d + eps);
  for (int i = 0; i < d; ++i) {
    float y = (x[i] - mean) * inv * w[i];
    if (b) y += b[i];
    out[i] = y;
  }
}

/* matmul_gated.wgsl:114-124 and laya.rs:1526-1539: erf by Abramowitz &
 * Stegun 7.1.26. */
static float laya_erf(float x) {
  const float s = x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : 0.0f);
  const float a = fabsf(x);
  const float t = 1.0f / (1.0f + 0.3275911f * a);
  const float poly =
      ((((1.061405429f * t - 1.453152027f) * t + 1.421413741f) * t - 0.284496736f) * t +
       0.254829592f) * t;
  return s * (1.0f - poly * expf(-a * a));
}

static float laya_gelu_erf(float x) { return 0.5f * x * (1.0f + laya_erf(x * 0.70710678118654752f)); }

/* attention_bi.wgsl:59-188 over the fused [t][q | k | v] rows (stride 3d):
 * a query sees the keys of its own sequence, within |dpos| <= window on
 * local layers (window 0 = all). */
static void laya_attention(const float* qkv, int t, int d, int heads, const int32_t* pos,
                           const int32_t* seq, int window, int mode, int threads, float* out) {
  const int hd = d / heads;
#pragma omp parallel for schedule(dynamic, 4) num_threads(threads)
  for (int i = 0; i < t; ++i) {
    float* sc = (float*)malloc(sizeof(float) * (size_t)t);
    int* idx = (int*)malloc(sizeof(int) * (size_t)t);
    float qh[1024], kj[1024];
    for (int hh = 0; hh < heads; ++hh) {
      const float* qr = qkv + (size_t)i * 3 * d + hh * hd;
      for (int dd = 0; dd < hd; ++dd) qh[dd] = mode == ORACLE_KERNEL ? round_f16(qr[dd]) : qr[dd];
      int n = 0;
      for (int j = 0; j < t; ++j) {
        if (seq[j] != seq[i]) continue;
        const int dist = pos[i] > pos[j] ? pos[i] - pos[j] : pos[j] - pos[i];
        if (window != 0 && dist > window) continue;
        const float* kr = qkv + (size_t)j * 3 * d + d + hh * hd;
        for (int dd = 0; dd < hd; ++dd) kj[dd] = mode == ORACLE_KERNEL ? round_f16(kr[dd]) : kr[dd];
        sc[n] = dot8(qh, kj, hd);
        idx[n++] = j;
      }
      float m = -INFINITY;
      for (int s = 0; s < n; ++s) m = fmaxf(m, sc[s]);
      float l = 0.0f;
      for (int s = 0; s < n; ++s) l += expf(sc[s] - m);
      float* o = out + (size_t)i * d + hh * hd;
      for (int dd = 0; dd < hd; ++dd) o[dd] = 0.0f;
      for (int s = 0; s < n; ++s) {
        const float p = expf(sc[s] - m) / l;
        const float* vr = qkv + (size_t)idx[s] * 3 * d + 2 * d + hh * hd;
        for (int dd = 0; dd < hd; ++dd) {
          const float vv = mode == ORACLE_KERNEL ? round_f16(vr[dd]) : vr[dd];
          o[dd] += p * vv;
        }
      }
    }
    free(sc);
    free(idx);
  }
}

int oracle_laya_hidden(const oracle_laya_config* cfg, const float* const* tensors,
                       size_t n_tensors, const uint32_t* ids, const int32_t* pos,
                       const int32_t* seq, const uint32_t* qtype, size_t t_, int mode,
                       int threads, float* x_out) {
  const int d = cfg->d, L = cfg->layers, heads = cfg->heads, ff = cfg->ff;
  const int hd = d / heads;
  const int t = (int)t_;
  if (t <= 0 || heads <= 0 || d % heads != 0 || hd > 1024) return -1;
  if (threads <= 0) {
#ifdef _OPENMP
    threads = omp_get_max_threads();
#else
    threads = 1;
#endif
  }
  /* Catalogue order of LayaConfig::tensors (laya.rs:265-313). */
  size_t ti = 0;
  int missing = 0;
#define NEXT() (ti < n_tensors && tensors[ti] ? tensors[ti++] : (missing = 1, (const float*)NULL))
  const float* embed = NEXT();
  const float* embed_norm = NEXT();
  const float* final_norm = NEXT();
  const float* type_emb = cfg->type_emb ? NEXT() : NULL;
  typedef struct { const float *attn_norm, *qkv, *o, *mlp_norm, *val, *gate, *wo; } enc_w;
  typedef struct {
    const float *n1w, *n1b, *in, *in_b, *out, *out_b, *n2w, *n2b, *l1, *l1_b, *l2, *l2_b;
  } head_w;
  enc_w* ew = (enc_w*)calloc((size_t)L, sizeof(enc_w));
  head_w* hw = (head_w*)calloc((size_t)(cfg->head_layers > 0 ? cfg->head_layers : 1), sizeof(head_w));
  for (int l = 0; l < L; ++l) {
    ew[l].attn_norm = l > 0 ? NEXT() : NULL;
    ew[l].qkv = NEXT();
    ew[l].o = NEXT();
    ew[l].mlp_norm = NEXT();
    ew[l].val = NEXT();
    ew[l].gate = NEXT();
    ew[l].wo = NEXT();
  }
  for (int h = 0; h < cfg->head_layers; ++h) {
    hw[h].n1w = NEXT(); hw[h].n1b = NEXT();
    hw[h].in = NEXT(); hw[h].in_b = NEXT();
    hw[h].out = NEXT(); hw[h].out_b = NEXT();
    hw[h].n2w = NEXT(); hw[h].n2b = NEXT();
    hw[h].l1 = NEXT(); hw[h].l1_b = NEXT();
    hw[h].l2 = NEXT(); hw[h].l2_b = NEXT();
  }
#undef NEXT
  const size_t T = (size_t)t;
  const int wide = ff > 4 * d ? ff : 4 * d;
  float* x = x_out;
  float* h = (float*)malloc(sizeof(float) * T * d);
  float* qkv = (float*)malloc(sizeof(float) * T * 3 * d);
  float* attn = (float*)malloc(sizeof(float) * T * d);
  float* a = (float*)malloc(sizeof(float) * T * d);
  float* g1 = (float*)malloc(sizeof(float) * T * wide);
  float* g2 = (float*)malloc(sizeof(float) * T * wide);
  int rc = 0;
  if (missing) {
    rc = -2;
    goto done;
  }

  /* embed (scale 1, laya.rs:1264-1268) into h, embed_norm -> x. */
  for (int i = 0; i < t; ++i) {
    memcpy(h + (size_t)i * d, embed + (size_t)ids[i] * d, sizeof(float) * d);
    laya_ln_row(h + (size_t)i * d, NULL, NULL, embed_norm, NULL, d, cfg->eps, x + (size_t)i * d);
  }
  for (int l = 0; l < L; ++l) {
    const enc_w* W = &ew[l];
    const int sliding = cfg->sliding[l];
    /* mm_qkv reads x on layer 0 (its norm is the embedding norm), h after. */
    linear_rows(l > 0 ? h : x, t, d, W->qkv, 3 * d, mode, qkv, threads);
    /* rope_bi.wgsl: whole-head rotation at the token's position, q * hd^-0.5. */
    const float theta = sliding ? cfg->theta_local : cfg->theta_global;
    const float scale = powf((float)hd, -0.5f);
    for (int i = 0; i < t; ++i)
      for (int hh = 0; hh < heads; ++hh)
        for (int dd = 0; dd < hd / 2; ++dd) {
          const float ang = (float)pos[i] * powf(theta, -(float)(2 * dd) / (float)hd);
          const float c = cosf(ang), s = sinf(ang);
          float* q = qkv + (size_t)i * 3 * d + hh * hd;
          float* k = q + d;
          const float qa = q[dd], qb = q[dd + hd / 2];
          q[dd] = (qa * c - qb * s) * scale;
          q[dd + hd / 2] = (qb * c + qa * s) * scale;
          const float ka = k[dd], kb = k[dd + hd / 2];
          k[dd] = ka * c - kb * s;
          k[dd + hd / 2] = kb * c + ka * s;
        }
    laya_attention(qkv, t, d, heads, pos, seq, sliding ? cfg->window : 0, mode, threads, attn);
    linear_rows(attn, t, d, W->o, d, mode, a, threads);
    /* add_o_norm: x += a, h = mlp_norm(x). */
    for (int i = 0; i < t; ++i)
      laya_ln_row(x + (size_t)i * d, a + (size_t)i * d, NULL, W->mlp_norm, NULL, d, cfg->eps,
                  h + (size_t)i * d);
    /* mm_wi: gelu_erf(h Wval^T) * (h Wgate^T). */
    linear_rows(h, t, d, W->val, ff, mode, g1, threads);
    linear_rows(h, t, d, W->gate, ff, mode, g2, threads);
    for (size_t k = 0; k < T * ff; ++k) g1[k] = laya_gelu_erf(g1[k]) * g2[k];
    linear_rows(g1, t, ff, W->wo, d, mode, a, threads);
    /* add_wo_norm: x += a, then the next layer's attn_norm into h, or the
     * final norm over x in place on the last layer. */
    for (int i = 0; i < t; ++i) {
      float* xi = x + (size_t)i * d;
      if (l + 1 < L) {
        laya_ln_row(xi, a + (size_t)i * d, NULL, ew[l + 1].attn_norm, NULL, d, cfg->eps,
                    h + (size_t)i * d);
      } else {
        float tmp[8192];
        laya_ln_row(xi, a + (size_t)i * d, NULL, final_norm, NULL, d, cfg->eps, tmp);
        memcpy(xi, tmp, sizeof(float) * d);
      }
    }
  }
  /* type_emb (embed.wgsl with residual = 1, scale 1). */
  if (type_emb)
    for (int i = 0; i < t; ++i)
      for (int dd = 0; dd < d; ++dd) x[(size_t)i * d + dd] += type_emb[(size_t)qtype[i] * d + dd];
  /* Decision-head layers (laya.rs:1316-1345). */
  for (int hl = 0; hl < cfg->head_layers; ++hl) {
    const head_w* W = &hw[hl];
    if (hl == 0)
      for (int i = 0; i < t; ++i) {
        float tmp[8192];
        memcpy(tmp, x + (size_t)i * d, sizeof(float) * d);
        laya_ln_row(tmp, NULL, NULL, W->n1w, W->n1b, d, cfg->eps, h + (size_t)i * d);
      }
    linear_rows(h, t, d, W->in, 3 * d, mode, qkv, threads);
    for (int i = 0; i < t; ++i)
      for (int c = 0; c < 3 * d; ++c) qkv[(size_t)i * 3 * d + c] += W->in_b[c];
    /* No RoPE and no query scale on the head's attention (laya.rs:1322-1327). */
    laya_attention(qkv, t, d, heads, pos, seq, 0, mode, threads, attn);
    linear_rows(attn, t, d, W->out, d, mode, a, threads);
    for (int i = 0; i < t; ++i)
      laya_ln_row(x + (size_t)i * d, a + (size_t)i * d, W->out_b, W->n2w, W->n2b, d, cfg->eps,
                  h + (size_t)i * d);
    linear_rows(h, t, d, W->l1, 4 * d, mode, g1, threads);
    for (int i = 0; i < t; ++i)
      for (int c = 0; c < 4 * d; ++c) {
        const float y = g1[(size_t)i * 4 * d + c] + W->l1_b[c];
        g1[(size_t)i * 4 * d + c] = y > 0.0f ? y : 0.0f;
      }
    linear_rows(g1, t, 4 * d, W->l2, d, mode, a, threads);
    if (hl + 1 == cfg->head_layers) {
      /* bias_act.wgsl with residual: x = (a + b) + x. */
      for (int i = 0; i < t; ++i)
        for (int c = 0; c < d; ++c) {
          float* xi = x + (size_t)i * d + c;
          *xi = (a[(size_t)i * d + c] + W->l2_b[c]) + *xi;
        }
    } else {
      for (int i = 0; i < t; ++i)
        laya_ln_row(x + (size_t)i * d, a + (size_t)i * d, W->l2_b, hw[hl + 1].n1w, hw[hl + 1].n1b,
                    d, cfg->eps, h + (size_t)i * d);
    }
  }
done:
  free(h);
  free(qkv);
  free(attn);
  free(a);
  free(g1);
  free(g2);
  free(ew);
  free(hw);
  return rc;
}

/* laya.rs:1500-1523: host LayerNorm, linear and softmax of the scorer. */
static void host_ln(const float* x, const float* w, const float* b, int n, float eps, float* out) {
  float s = 0.0f;
  for (int i = 0; i < n; ++i) s += x[i];
  const float mean = s / (float)n;
  float v = 0.0f;
  for (int i = 0; i < n; ++i) v += (x[i] - mean) * (x[i] - mean);
  v /= (float)n;
  const float inv = 1.0f / sqrtf(v + eps);
  for (int i = 0; i < n; ++i) out[i] = (x[i] - mean) * inv * w[i] + b[i];
}

static float host_dot(const float* a, const float* b, int n) {
  float s = 0.0f;
  for (int i = 0; i < n; ++i) s += a[i] * b[i];
  return s;
}

static void host_softmax(const float* z, int n, float* out) {
  float m = -INFINITY;
  for (int i = 0; i < n; ++i) m = fmaxf(m, z[i]);
  float s = 0.0f;
  for (int i = 0; i < n; ++i) {
    out[i] = expf(z[i] - m);
    s += out[i];
  }
  for (int i = 0; i < n; ++i) out[i] /= s;
}

int oracle_laya_score(const float* rows, int k, int d, float eps, const float* const* w,
                      int act_hidden, int act_out, float* logits, float* act_prob) {
  /* w: scorer.norm_w, norm_b, l1, l1_b, l2, l2_b, then act.l1, l1_b, l2, l2_b. */
  if (k < 1 || d > 8192) return -1;
  float z[8192], y[8192];
  for (int o = 0; o < k; ++o) {
    host_ln(rows + (size_t)(o + 1) * d, w[0], w[1], d, eps, z);
    for (int r = 0; r < d; ++r) y[r] = laya_gelu_erf(host_dot(w[2] + (size_t)r * d, z, d) + w[3][r]);
    logits[o] = host_dot(y, w[4], d) + w[5][0];
  }
  if (act_out <= 0) return 0;
  const int kk = k > 2 ? k : 2;
  float* padded = (float*)malloc(sizeof(float) * (size_t)kk);
  float* p = (float*)malloc(sizeof(float) * (size_t)kk);
  for (int i = 0; i < kk; ++i) padded[i] = i < k ? logits[i] : -1e4f;
  host_softmax(padded, kk, p);
  float ent = 0.0f;
  for (int i = 0; i < kk; ++i) ent += p[i] * logf(p[i] > 1e-9f ? p[i] : 1e-9f);
  ent = -ent / logf((float)kk);
  /* top1 / top2 of the sorted probabilities. */
  float top1 = -INFINITY, top2 = -INFINITY;
  for (int i = 0; i < kk; ++i) {
    if (p[i] > top1) {
      top2 = top1;
      top1 = p[i];
    } else if (p[i] > top2) {
      top2 = p[i];
    }
  }
  float* pooled = (float*)malloc(sizeof(float) * (size_t)(d + 4));
  memcpy(pooled, rows, sizeof(float) * d);
  pooled[d] = top1;
  pooled[d + 1] = top1 - top2;
  pooled[d + 2] = ent;
  pooled[d + 3] = (float)kk / 255.0f;
  float* ah = (float*)malloc(sizeof(float) * (size_t)act_hidden);
  for (int r = 0; r < act_hidden; ++r)
    ah[r] = laya_gelu_erf(host_dot(w[6] + (size_t)r * (d + 4), pooled, d + 4) + w[7][r]);
  float* ao = (float*)malloc(sizeof(float) * (size_t)act_out);
  float* ap = (float*)malloc(sizeof(float) * (size_t)act_out);
  for (int r = 0; r < act_out; ++r) ao[r] = host_dot(w[8] + (size_t)r * act_hidden, ah, act_hidden) + w[9][r];
  host_softmax(ao, act_out, ap);
  *act_prob = ap[0];
  free(padded);
  free(p);
  free(pooled);
  free(ah);
  free(ao);
  free(ap);
  return 0;
}
