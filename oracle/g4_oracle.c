/*
 * g4_oracle.c -- CPU restatement of gemma4.kt's hot-path kernels.
 * TEST INFRASTRUCTURE ONLY (see g4_oracle.h).  Build: oracle/Makefile
 * (gcc -O2 -ffp-contract=off).
 *
 * Reference paths below are relative to
 * lib/src/main/kotlin/io/github/lbenedetto/internal/.
 */
#include "g4_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#define LANES 16 /* 512-bit FloatVector species, FloatTensorHelpers.kt:9-29 */
#define QK_K 256 /* GGMLType.kt:5 */
#define JAVA_PI 3.141592653589793 /* Math.PI */

int o_block_size(int type) {
  switch (type) {
    case O_Q4_0:
    case O_Q4_1:
    case O_Q5_1:
    case O_Q8_0:
    case O_MXFP4: return 32;  /* QK_MXFP4, GGMLType.kt:6 */
    case O_Q4_K:
    case O_Q5_K:
    case O_Q6_K: return QK_K;
    default: return 1;
  }
}

int o_type_size(int type) {
  switch (type) {
    case O_F32: return 4;
    case O_F16: return 2;
    case O_BF16: return 2;
    case O_Q4_0: return 18;   /* GGMLType.kt:18 */
    case O_Q4_1: return 20;   /* GGMLType.kt:19 */
    case O_Q5_1: return 24;   /* GGMLType.kt:23 */
    case O_Q8_0: return 34;   /* GGMLType.kt:24 */
    case O_Q4_K: return 144;  /* GGMLType.kt:28 */
    case O_Q5_K: return 176;  /* GGMLType.kt:29 */
    case O_Q6_K: return 210;  /* GGMLType.kt:30 */
    case O_MXFP4: return 17;  /* GGMLType.kt:55 */
    default: return 0;
  }
}

static inline float bits_to_f32(uint32_t b) {
  float f;
  memcpy(&f, &b, 4);
  return f;
}

static inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* Exact binary16 -> binary32.  Same bit construction as
 * Q6_KFloatTensor.fp16ToFloatNoIntrinsic (Q6_KFloatTensor.kt:87-109), which
 * agrees with Float.float16ToFloat for every non-NaN input. */
float o_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  if (exp == 0) {
    if (man == 0) return bits_to_f32(sign);
    int e = 127 - 15 + 1;
    while ((man & 0x400u) == 0) {
      man <<= 1;
      e--;
    }
    man &= 0x3FFu;
    return bits_to_f32(sign | ((uint32_t)e << 23) | (man << 13));
  }
  if (exp == 0x1F) return bits_to_f32(sign | 0x7F800000u | (man << 13));
  return bits_to_f32(sign | ((exp + (127 - 15)) << 23) | (man << 13));
}

static inline float rd_f16(const uint8_t *p) { return o_f16_to_f32(rd16(p)); }

/* Q4_KFloatTensor.getScaleMinK4 (Q4_KFloatTensor.kt:70-84) */
static int scale_min_k4(int j, const uint8_t *s, int is_min) {
  if (j < 4) return s[is_min ? j + 4 : j] & 63;
  int low = is_min ? (s[j + 4] >> 4) : (s[j + 4] & 0xF);
  int high = (s[is_min ? j : j - 4] >> 6) & 0x3;
  return low | (high << 4);
}

float o_get(int type, const uint8_t *base, int64_t index) {
  switch (type) {
    case O_F32: { /* F32FloatTensor.kt:18-20 */
      float f;
      memcpy(&f, base + index * 4, 4);
      return f;
    }
    case O_F16:
      return rd_f16(base + index * 2);
    case O_BF16: /* BF16FloatTensor.kt:20-24 */
      return bits_to_f32((uint32_t)rd16(base + index * 2) << 16);
    case O_Q8_0: { /* Q8_0FloatTensor.kt:21-28: quant * scale, one rounding */
      int64_t b = index / 32, w = index % 32;
      const uint8_t *blk = base + b * 34;
      float scale = rd_f16(blk);
      return (float)(int8_t)blk[2 + w] * scale;
    }
    case O_Q4_K: { /* Q4_KFloatTensor.kt:23-55 */
      int64_t b = index / QK_K;
      int within = (int)(index % QK_K);
      const uint8_t *blk = base + b * 144;
      float d = rd_f16(blk), dmin = rd_f16(blk + 2);
      const uint8_t *sc = blk + 4, *qs = blk + 16;
      int group = within / 64, in_group = within % 64;
      int sub, nib, high;
      if (in_group < 32) {
        sub = group * 2;
        nib = in_group;
        high = 0;
      } else {
        sub = group * 2 + 1;
        nib = in_group - 32;
        high = 1;
      }
      int s = scale_min_k4(sub, sc, 0), m = scale_min_k4(sub, sc, 1);
      uint8_t byte = qs[group * 32 + nib];
      int q = high ? (byte >> 4) & 0xF : byte & 0xF;
      /* d * sc * quant - dmin * m: ((d*sc)*q) - (dmin*m), each op rounded */
      float t = d * (float)s;
      t = t * (float)q;
      float u = dmin * (float)m;
      return t - u;
    }
    case O_Q4_0: { /* Q4_0FloatTensor.kt:20-38: (q - 8) * scale */
      const uint8_t *blk = base + (index / 32) * 18;
      int w = (int)(index % 32);
      int q = w < 16 ? (blk[2 + w] & 0x0F) : ((blk[2 + w - 16] >> 4) & 0x0F);
      return (float)(q - 8) * rd_f16(blk);
    }
    case O_Q4_1: { /* Q4_1FloatTensor.kt:22-41: delta * quant + min, two roundings */
      const uint8_t *blk = base + (index / 32) * 20;
      int w = (int)(index % 32);
      int q = w < 16 ? (blk[4 + w] & 0x0F) : ((blk[4 + w - 16] >> 4) & 0x0F);
      float t = rd_f16(blk) * (float)q;
      return t + rd_f16(blk + 2);
    }
    case O_Q5_1: { /* Q5_1FloatTensor.kt:20-51: q * d + m, fifth bit from the 32-bit qh */
      const uint8_t *blk = base + (index / 32) * 24;
      int w = (int)(index % 32);
      uint32_t qh = (uint32_t)blk[4] | ((uint32_t)blk[5] << 8) | ((uint32_t)blk[6] << 16) | ((uint32_t)blk[7] << 24);
      int nib, xh;
      if (w < 16) {
        nib = blk[8 + w] & 0x0F;
        xh = (int)((qh >> w) << 4) & 0x10;
      } else {
        nib = (blk[8 + w - 16] >> 4) & 0x0F;
        xh = (int)(qh >> (w - 16 + 12)) & 0x10;
      }
      float t = (float)(nib | xh) * rd_f16(blk);
      return t + rd_f16(blk + 2);
    }
    case O_Q5_K: { /* Q5_KFloatTensor.kt:23-50: d * sc * quant - dmin * m, quant = nibble | qh bit << 4 */
      const uint8_t *blk = base + (index / QK_K) * 176;
      int within = (int)(index % QK_K);
      float d = rd_f16(blk), dmin = rd_f16(blk + 2);
      int group = within / 64, in_group = within % 64, high = in_group >= 32, l = high ? in_group - 32 : in_group;
      int sub = group * 2 + high;
      int sc = scale_min_k4(sub, blk + 4, 0), m = scale_min_k4(sub, blk + 4, 1);
      uint8_t qb = blk[48 + group * 32 + l];
      int nib = high ? ((qb >> 4) & 0xF) : (qb & 0xF);
      int hbit = (blk[16 + l] >> (2 * group + high)) & 1;
      float t = d * (float)sc;
      t = t * (float)(nib | (hbit << 4));
      float u = dmin * (float)m;
      return t - u;
    }
    case O_MXFP4: { /* MXFP4FloatTensor.kt:22-36,49,209-216: E2M1 value * 2^(e8m0 - 128) */
      static const int vals[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};
      const uint8_t *blk = base + (index / 32) * 17;
      int w = (int)(index % 32);
      int e = blk[0];
      uint32_t bits = e < 2 ? (0x00200000u << e) : ((uint32_t)(e - 1) << 23);
      float dd = bits_to_f32(bits);
      int packed = blk[1 + (w & 0x0F)];
      int nib = w < 16 ? (packed & 0x0F) : ((packed >> 4) & 0x0F);
      return (float)vals[nib] * dd;
    }
    case O_Q6_K: { /* Q6_KFloatTensor.kt:26-73 */
      int64_t b = index / QK_K;
      int within = (int)(index % QK_K);
      const uint8_t *blk = base + b * 210;
      const uint8_t *qh = blk + 128;
      const int8_t *sc = (const int8_t *)(blk + 192);
      float d = rd_f16(blk + 208);
      int half = within / 128, rem = within % 128, sub32 = rem / 32, l = rem % 32;
      const uint8_t *ql = blk + half * 64;
      const uint8_t *qhb = qh + half * 32;
      int nib, shift;
      switch (sub32) {
        case 0: nib = ql[l] & 0xF; shift = 0; break;
        case 1: nib = ql[32 + l] & 0xF; shift = 2; break;
        case 2: nib = (ql[l] >> 4) & 0xF; shift = 4; break;
        default: nib = (ql[32 + l] >> 4) & 0xF; shift = 6; break;
      }
      int hb = (qhb[l] >> shift) & 3;
      int q6 = (nib | (hb << 4)) - 32;
      int s = sc[half * 8 + sub32 * 2 + l / 16];
      float t = d * (float)s;
      return t * (float)q6;
    }
    default:
      return NAN;
  }
}

void o_dequant(int type, const uint8_t *base, int64_t offset, int64_t n, float *out) {
  for (int64_t i = 0; i < n; i++) out[i] = o_get(type, base, offset + i);
}

/* FloatTensorHelpers.scalarDot (FloatTensorHelpers.kt:65-71): sequential,
 * product rounded then added. */
float o_scalar_dot(int type, const uint8_t *base, int64_t this_offset, const float *x, int size) {
  float r = 0.0f;
  for (int j = 0; j < size; j++) {
    float p = o_get(type, base, this_offset + j) * x[j];
    r = r + p;
  }
  return r;
}

/* FloatVector.reduceLanes(ADD): the JVM leaves the order unspecified; the
 * oracle uses a fixed pairwise tree. */
static float reduce_lanes(const float *v) {
  float t[LANES];
  memcpy(t, v, sizeof t);
  for (int w = LANES / 2; w >= 1; w >>= 1)
    for (int i = 0; i < w; i++) t[i] = t[i] + t[i + w];
  return t[0];
}

/* Alignment head shared by the quantized vectorDots (e.g. Q8_0FloatTensor.kt:50-54):
 * elements before the next block boundary go through scalarDot. */
static int head_len(int64_t this_offset, int bs, int size) {
  int64_t rem = this_offset % bs;
  int h = rem == 0 ? 0 : (int)(bs - rem);
  return h < size ? h : size;
}

/* Q8_0FloatTensor.vectorDot, 512-bit branch (Q8_0FloatTensor.kt:39-78,132-141) */
static float dot_q8_0(const uint8_t *base, int64_t off, const float *x, int size) {
  float result = 0.0f;
  int j = head_len(off, 32, size);
  if (j > 0) result += o_scalar_dot(O_Q8_0, base, off, x, j);
  float acc[LANES] = {0};
  const uint8_t *blk = base + (off + j) / 32 * 34;
  int upper = j + (size - j) / 32 * 32;
  for (; j < upper; j += 32, blk += 34) {
    float d = rd_f16(blk);
    const int8_t *q = (const int8_t *)(blk + 2);
    for (int l = 0; l < LANES; l++) {
      float s0 = x[j + l] * (float)q[l];
      float s1 = x[j + LANES + l] * (float)q[LANES + l];
      acc[l] = fmaf(s0 + s1, d, acc[l]);
    }
  }
  result += reduce_lanes(acc);
  if (j < size) result += o_scalar_dot(O_Q8_0, base, off + j, x + j, size - j);
  return result;
}

/* Q4_KFloatTensor.vectorDot, 512-bit branch (Q4_KFloatTensor.kt:86-148,196-206) */
static float dot_q4_k(const uint8_t *base, int64_t off, const float *x, int size) {
  float result = 0.0f;
  int j = head_len(off, QK_K, size);
  if (j > 0) result += o_scalar_dot(O_Q4_K, base, off, x, j);
  float v1[LANES] = {0}, v2[LANES] = {0};
  const uint8_t *blk = base + (off + j) / QK_K * 144;
  int upper = j + (size - j) / QK_K * QK_K;
  for (; j < upper; j += QK_K, blk += 144) {
    float d = rd_f16(blk), dmin = rd_f16(blk + 2);
    const uint8_t *sc = blk + 4, *qs = blk + 16;
    for (int g = 0; g < 4; g++) {
      float d1 = d * (float)scale_min_k4(2 * g, sc, 0);
      float negm1 = -(dmin * (float)scale_min_k4(2 * g, sc, 1));
      float d2 = d * (float)scale_min_k4(2 * g + 1, sc, 0);
      float negm2 = -(dmin * (float)scale_min_k4(2 * g + 1, sc, 1));
      for (int c = 0; c < 2; c++) {
        const uint8_t *w = qs + g * 32 + c * 16;
        const float *xlo = x + j + g * 64 + c * 16;
        const float *xhi = x + j + g * 64 + 32 + c * 16;
        for (int l = 0; l < LANES; l++) {
          float lo = (float)(w[l] & 0xF), hi = (float)(w[l] >> 4);
          v1[l] = fmaf(fmaf(lo, d1, negm1), xlo[l], v1[l]);
          v2[l] = fmaf(fmaf(hi, d2, negm2), xhi[l], v2[l]);
        }
      }
    }
  }
  float s[LANES];
  for (int l = 0; l < LANES; l++) s[l] = v1[l] + v2[l];
  result += reduce_lanes(s);
  if (j < size) result += o_scalar_dot(O_Q4_K, base, off + j, x + j, size - j);
  return result;
}

/* Q6_KFloatTensor.vectorDot, 512-bit branch (Q6_KFloatTensor.kt:111-205,239-249) */
static float dot_q6_k(const uint8_t *base, int64_t off, const float *x, int size) {
  float result = 0.0f;
  int j = head_len(off, QK_K, size);
  if (j > 0) result += o_scalar_dot(O_Q6_K, base, off, x, j);
  float acc[LANES] = {0};
  const uint8_t *blk = base + (off + j) / QK_K * 210;
  int upper = j + (size - j) / QK_K * QK_K;
  for (; j < upper; j += QK_K, blk += 210) {
    const int8_t *sc = (const int8_t *)(blk + 192);
    float d = rd_f16(blk + 208);
    for (int h = 0; h < 2; h++) {
      const uint8_t *ql = blk + h * 64, *qh = blk + 128 + h * 32;
      const float *xb = x + j + h * 128;
      for (int c = 0; c < 2; c++) {
        const uint8_t *a = ql + c * 16, *b = ql + 32 + c * 16, *hv = qh + c * 16;
        float ds0 = d * (float)sc[h * 8 + c];
        float ds1 = d * (float)sc[h * 8 + 2 + c];
        float ds2 = d * (float)sc[h * 8 + 4 + c];
        float ds3 = d * (float)sc[h * 8 + 6 + c];
        for (int l = 0; l < LANES; l++) {
          int q0 = (int)(int8_t)(uint8_t)(((a[l] & 0xF) | ((hv[l] & 3) << 4)) - 32);
          int q1 = (int)(int8_t)(uint8_t)(((b[l] & 0xF) | (((hv[l] >> 2) & 3) << 4)) - 32);
          int q2 = (int)(int8_t)(uint8_t)(((a[l] >> 4) | (((hv[l] >> 4) & 3) << 4)) - 32);
          int q3 = (int)(int8_t)(uint8_t)(((b[l] >> 4) | (((hv[l] >> 6) & 3) << 4)) - 32);
          acc[l] = fmaf((float)q0 * ds0, xb[c * 16 + l], acc[l]);
          acc[l] = fmaf((float)q1 * ds1, xb[32 + c * 16 + l], acc[l]);
          acc[l] = fmaf((float)q2 * ds2, xb[64 + c * 16 + l], acc[l]);
          acc[l] = fmaf((float)q3 * ds3, xb[96 + c * 16 + l], acc[l]);
        }
      }
    }
  }
  result += reduce_lanes(acc);
  if (j < size) result += o_scalar_dot(O_Q6_K, base, off + j, x + j, size - j);
  return result;
}

/* BF16FloatTensor.vectorDot (BF16FloatTensor.kt:35-74) and
 * F32FloatTensor.vectorDot (F32FloatTensor.kt:37-66): plain 16-lane fma over
 * loopBound(size), then a sequential tail added onto the reduced sum. */
static float dot_wide(int type, const uint8_t *base, int64_t off, const float *x, int size) {
  float acc[LANES] = {0};
  int upper = size / LANES * LANES;
  for (int i = 0; i < upper; i += LANES)
    for (int l = 0; l < LANES; l++) acc[l] = fmaf(o_get(type, base, off + i + l), x[i + l], acc[l]);
  float result = reduce_lanes(acc);
  if (type == O_BF16) {
    if (upper < size) result += o_scalar_dot(type, base, off + upper, x + upper, size - upper);
  } else {
    for (int i = upper; i < size; i++) {
      float p = o_get(type, base, off + i) * x[i];
      result = result + p;
    }
  }
  return result;
}

float o_vector_dot(int type, const uint8_t *base, int64_t this_offset, const float *x, int size) {
  switch (type) {
    case O_Q8_0: return dot_q8_0(base, this_offset, x, size);
    case O_Q4_K: return dot_q4_k(base, this_offset, x, size);
    case O_Q6_K: return dot_q6_k(base, this_offset, x, size);
    case O_BF16:
    case O_F32: return dot_wide(type, base, this_offset, x, size);
    default: return o_scalar_dot(type, base, this_offset, x, size);
  }
}

typedef struct {
  int type, dim1, vector, r0, r1;
  const uint8_t *base;
  int64_t off;
  const float *x;
  float *out;
} mm_job;

static void *mm_worker(void *p) {
  mm_job *jb = (mm_job *)p;
  for (int i = jb->r0; i < jb->r1; i++) {
    int64_t o = jb->off + (int64_t)i * jb->dim1;
    jb->out[i] = jb->vector ? o_vector_dot(jb->type, jb->base, o, jb->x, jb->dim1)
                            : o_scalar_dot(jb->type, jb->base, o, jb->x, jb->dim1);
  }
  return NULL;
}

void o_matmul(int type, const uint8_t *base, int64_t this_offset, const float *x, float *out,
              int dim0, int dim1, int nthreads, int vector) {
  if (nthreads < 1) nthreads = 1;
  if (nthreads > dim0) nthreads = dim0 > 0 ? dim0 : 1;
  mm_job jobs[256];
  pthread_t th[256];
  if (nthreads > 256) nthreads = 256;
  for (int t = 0; t < nthreads; t++) {
    jobs[t] = (mm_job){type, dim1, vector, (int)((int64_t)dim0 * t / nthreads),
                       (int)((int64_t)dim0 * (t + 1) / nthreads), base, this_offset, x, out};
  }
  for (int t = 1; t < nthreads; t++) pthread_create(&th[t], NULL, mm_worker, &jobs[t]);
  mm_worker(&jobs[0]);
  for (int t = 1; t < nthreads; t++) pthread_join(th[t], NULL);
}

/* Llama.gelu (Llama.kt:23-25): evaluated in double, rounded to float */
float o_gelu(float x) {
  double xd = (double)x;
  double inner = sqrt(2.0 / JAVA_PI) * (xd + 0.044715 * pow(xd, 3.0));
  return (float)(0.5 * xd * (1.0 + tanh(inner)));
}

/* Llama.rmsnorm (Llama.kt:27-37): sequential float sum of squares, 1/sqrt in
 * double, out[i] = w[i] * (ss * x[i]).  out may alias x. */
void o_rmsnorm(float *out, const float *x, const float *w, int size, float eps) {
  float ss = 0.0f;
  for (int i = 0; i < size; i++) {
    float sq = x[i] * x[i];
    ss = ss + sq;
  }
  ss = ss / (float)size;
  ss = ss + eps;
  ss = (float)(1.0 / sqrt((double)ss));
  for (int i = 0; i < size; i++) {
    float t = ss * x[i];
    out[i] = w[i] * t;
  }
}

/* MutableFloatTensor.softmaxInPlace (MutableFloatTensor.kt:54-59) */
void o_softmax(float *x, int n) {
  float mx = -INFINITY;
  for (int i = 0; i < n; i++) mx = fmaxf(mx, x[i]); /* Math::max */
  for (int i = 0; i < n; i++) x[i] = (float)exp((double)(x[i] - mx));
  float sum = 0.0f;
  for (int i = 0; i < n; i++) sum = sum + x[i];
  for (int i = 0; i < n; i++) x[i] = x[i] / sum;
}

/* Smallest routing margin seen since the last reset: the gap between the
 * k-th and (k+1)-th largest router probability of a token.  Test
 * infrastructure: a fixture whose margin is at the level of fp32 rounding
 * (~1e-7) cannot pin an expert choice, since any implementation within the
 * tolerance may take the other expert there. */
static double g_topk_margin = INFINITY;

void o_reset_topk_margin(void) { g_topk_margin = INFINITY; }
double o_topk_margin(void) { return g_topk_margin; }

void o_note_topk_margin(const float *probs, int n, int k) {
  if (k <= 0 || k >= n || k > 64) return;
  float top[65]; /* the k+1 largest so far, descending */
  int m = 0;
  for (int e = 0; e < n; e++) {
    float v = probs[e];
    if (m == k + 1 && !(v > top[k])) continue;
    int i = m < k + 1 ? m++ : k; /* slot to fill, then move up */
    while (i > 0 && top[i - 1] < v) {
      top[i] = top[i - 1];
      i--;
    }
    top[i] = v;
  }
  double gap = (double)top[k - 1] - (double)top[k];
  if (gap < g_topk_margin) g_topk_margin = gap;
}

/* Llama.kt:276-293 */
void o_topk(float *probs, int n, int k, int32_t *idx, float *val) {
  for (int ki = 0; ki < k; ki++) {
    int best = 0;
    float bv = -INFINITY;
    for (int e = 0; e < n; e++) {
      if (probs[e] > bv) {
        bv = probs[e];
        best = e;
      }
    }
    idx[ki] = best;
    val[ki] = bv;
    probs[best] = -INFINITY;
  }
}

/* Router input and logits, Llama.kt:257-270 */
void o_moe_router_logits(const o_moe_weights *w, const float *x, float *logits) {
  int dim = w->dim;
  float ss = 0.0f;
  for (int i = 0; i < dim; i++) {
    float sq = x[i] * x[i];
    ss = ss + sq;
  }
  ss = ss / (float)dim;
  ss = ss + w->eps;
  float rms = (float)(1.0 / sqrt((double)ss)) / (float)sqrt((double)dim);
  float *xr = (float *)malloc(sizeof(float) * dim);
  for (int i = 0; i < dim; i++) {
    float t = x[i] * rms;
    xr[i] = t * w->gate_inp_scale[i];
  }
  for (int e = 0; e < w->n_expert; e++)
    logits[e] = o_vector_dot(O_F32, w->gate_inp, (int64_t)e * dim, xr, dim);
  free(xr);
}

void o_moe_token(const o_moe_weights *w, const float *x, float *out, int32_t *topk_idx,
                 float *topk_prob, float *router_logits_out, int nthreads) {
  int dim = w->dim, ff = w->expert_ff, gu = 2 * ff;
  float *moe_in = (float *)malloc(sizeof(float) * dim);
  float *probs = (float *)malloc(sizeof(float) * w->n_expert);
  float *gate_up = (float *)malloc(sizeof(float) * gu);
  float *down = (float *)malloc(sizeof(float) * dim);
  /* moeInput = rmsnorm(x, pre_ffw_norm_2), Llama.kt:248-254 */
  o_rmsnorm(moe_in, x, w->pre_ffw_norm_2, dim, w->eps);
  o_moe_router_logits(w, x, probs);
  if (router_logits_out) memcpy(router_logits_out, probs, sizeof(float) * w->n_expert);
  o_softmax(probs, w->n_expert); /* Llama.kt:273 */
  o_note_topk_margin(probs, w->n_expert, w->n_used);
  o_topk(probs, w->n_expert, w->n_used, topk_idx, topk_prob);
  for (int i = 0; i < dim; i++) out[i] = 0.0f; /* Llama.kt:298 */
  for (int ki = 0; ki < w->n_used; ki++) {       /* Llama.kt:300-337 */
    int e = topk_idx[ki];
    float prob = topk_prob[ki];
    float down_scale = w->down_exps_scale[e];
    int64_t gu_off = (int64_t)e * gu * dim;
    o_matmul(w->gate_up_type, w->gate_up_exps, gu_off, moe_in, gate_up, gu, dim, nthreads, 1);
    for (int i = 0; i < ff; i++) gate_up[i] = o_gelu(gate_up[i]);
    for (int i = 0; i < ff; i++) gate_up[i] = gate_up[i] * gate_up[ff + i];
    int64_t dn_off = (int64_t)e * dim * ff;
    o_matmul(w->down_type, w->down_exps, dn_off, gate_up, down, dim, ff, nthreads, 1);
    float fw = prob * down_scale;
    for (int i = 0; i < dim; i++) {
      float p = fw * down[i];
      out[i] = p + out[i];
    }
  }
  if (w->post_ffw_norm_2) o_rmsnorm(out, out, w->post_ffw_norm_2, dim, w->eps); /* Llama.kt:340-346 */
  free(moe_in);
  free(probs);
  free(gate_up);
  free(down);
}

/* ====================================================================== */
/* Whole-model forward, Llama.kt:105-408                                   */
/* ====================================================================== */

/* RotaryPositionEmbeddings.kt:8-27 (freq_factors == NULL) and :29-53 */
void o_rope_table(int ctx_len, int head_size, double theta, const float *freq_factors, float *cr, float *ci) {
  int half = head_size / 2;
  int64_t n = 0;
  for (int pos = 0; pos < ctx_len; pos++) {
    for (int i = 0; i < half; i++) {
      float value;
      if (freq_factors) {
        float base = (float)(1.0 / pow(theta, (2.0 * i) / head_size));
        value = (float)pos * base;
        value = value / freq_factors[i];
      } else {
        /* i0 = 2*i walks the head in steps of 2: theta^(i0 / headSize) */
        float freq = (float)(1.0 / pow(theta, (double)(2 * i) / (double)head_size));
        value = (float)pos * freq;
      }
      cr[n] = (float)cos((double)value);
      ci[n] = (float)sin((double)value);
      n++;
    }
  }
}

struct o_state {
  float *x, *xb, *xbk, *xb2, *hb, *hb2, *q, *k, *v, *att, *logits;
  float *moe_out;
  float **key_cache, **value_cache; /* [n_layer_kv_from_start][ctx * kvDim] */
  int n_kv_layers;
  float *cr_full, *ci_full, *cr_swa, *ci_swa;
};

static int head_size_of(const o_model *m, int l) { return m->is_swa[l] ? m->head_size_swa : m->head_size_full; }
static int kv_dim_of(const o_model *m, int l) { return m->n_kv_heads[l] * head_size_of(m, l); }

o_state *o_state_new(const o_model *m) {
  o_state *s = (o_state *)calloc(1, sizeof(o_state));
  int max_q = m->n_heads * (m->head_size_full > m->head_size_swa ? m->head_size_full : m->head_size_swa);
  int max_kv = 0, max_ff = 0;
  for (int l = 0; l < m->n_layers; l++) {
    if (kv_dim_of(m, l) > max_kv) max_kv = kv_dim_of(m, l);
    if (m->ff[l] > max_ff) max_ff = m->ff[l];
  }
  s->x = (float *)calloc(m->dim, 4);
  s->xb = (float *)calloc(m->dim, 4);
  s->xbk = (float *)calloc(max_q, 4);
  s->xb2 = (float *)calloc(m->dim, 4);
  s->hb = (float *)calloc(max_ff > 0 ? max_ff : 1, 4);
  s->hb2 = (float *)calloc(max_ff > 0 ? max_ff : 1, 4);
  s->q = (float *)calloc(max_q, 4);
  s->k = (float *)calloc(max_kv, 4);
  s->v = (float *)calloc(max_kv, 4);
  s->att = (float *)calloc((size_t)m->n_heads * m->ctx_len, 4);
  s->logits = (float *)calloc(m->vocab, 4);
  s->moe_out = (float *)calloc(m->dim, 4);
  int nkv = m->n_layer_kv_from_start;
  s->n_kv_layers = nkv;
  s->key_cache = (float **)calloc(nkv, sizeof(float *));
  s->value_cache = (float **)calloc(nkv, sizeof(float *));
  for (int l = 0; l < nkv; l++) {
    s->key_cache[l] = (float *)calloc((size_t)m->ctx_len * kv_dim_of(m, l), 4);
    s->value_cache[l] = (float *)calloc((size_t)m->ctx_len * kv_dim_of(m, l), 4);
  }
  size_t hf = (size_t)m->ctx_len * (m->head_size_full / 2), hs = (size_t)m->ctx_len * (m->head_size_swa / 2);
  s->cr_full = (float *)malloc(hf * 4);
  s->ci_full = (float *)malloc(hf * 4);
  s->cr_swa = (float *)malloc(hs * 4);
  s->ci_swa = (float *)malloc(hs * 4);
  /* ModelLoader.loadWeights (ModelLoader.kt:154-166) */
  o_rope_table(m->ctx_len, m->head_size_swa, (double)m->rope_theta_swa, NULL, s->cr_swa, s->ci_swa);
  o_rope_table(m->ctx_len, m->head_size_full, (double)m->rope_theta, m->rope_freqs, s->cr_full, s->ci_full);
  return s;
}

void o_state_free(o_state *s) {
  if (!s) return;
  free(s->x); free(s->xb); free(s->xbk); free(s->xb2); free(s->hb); free(s->hb2);
  free(s->q); free(s->k); free(s->v); free(s->att); free(s->logits); free(s->moe_out);
  free(s->cr_full); free(s->ci_full); free(s->cr_swa); free(s->ci_swa);
  for (int l = 0; l < s->n_kv_layers; l++) {
    free(s->key_cache[l]);
    free(s->value_cache[l]);
  }
  free(s->key_cache);
  free(s->value_cache);
  free(s);
}

/* Llama.kt:39-59: rmsnorm with offsets: out = (weight * ss) * x, left to right */
static void rmsnorm_off(float *out, const float *x, const float *w, int size, float eps) {
  float ss = 0.0f;
  for (int i = 0; i < size; i++) {
    float sq = x[i] * x[i];
    ss = ss + sq;
  }
  ss = ss / (float)size;
  ss = ss + eps;
  ss = (float)(1.0 / sqrt((double)ss));
  for (int i = 0; i < size; i++) {
    float t = w[i] * ss;
    out[i] = t * x[i];
  }
}

/* Llama.kt:62-81: bare RMS norm */
static void rmsnorm_noweight(float *out, const float *x, int size, float eps) {
  float ss = 0.0f;
  for (int i = 0; i < size; i++) {
    float sq = x[i] * x[i];
    ss = ss + sq;
  }
  ss = ss / (float)size;
  ss = ss + eps;
  ss = (float)(1.0 / sqrt((double)ss));
  for (int i = 0; i < size; i++) out[i] = ss * x[i];
}

/* Llama.kt:83-103 (NeoX pairs ic, ic + halfHead) */
static void rope(float *v, int h, int head_size, const float *fr, const float *fi, int position) {
  int half = head_size / 2, po = h * head_size;
  for (int ic = 0; ic < half; ic++) {
    float fcr = fr[(size_t)position * half + ic], fci = fi[(size_t)position * half + ic];
    float v0 = v[po + ic], v1 = v[po + ic + half];
    float a = v0 * fcr, b = v1 * fci;
    float c = v0 * fci, d = v1 * fcr;
    v[po + ic] = a - b;
    v[po + ic + half] = c + d;
  }
}

/* llama.VectorBitSize=0 runs every dot product through scalarDot
 * (FloatTensorHelpers.kt:9-21, USE_VECTOR_API false); o_set_vector_api(0)
 * selects that mode for the whole-model forward. */
static int g_vector_api = 1;
void o_set_vector_api(int on) { g_vector_api = on != 0; }

/* ArrayFloatTensor.dot (ArrayFloatTensor.kt:48-87): 16-lane fma, reduceLanes,
 * scalar tail; scalarDot when the Vector API is off */
static float array_dot(const float *a, const float *b, int size) {
  if (!g_vector_api) {
    float r = 0.0f;
    for (int i = 0; i < size; i++) {
      float p = a[i] * b[i];
      r = r + p;
    }
    return r;
  }
  float acc[LANES] = {0};
  int upper = size / LANES * LANES;
  for (int i = 0; i < upper; i += LANES)
    for (int l = 0; l < LANES; l++) acc[l] = fmaf(a[i + l], b[i + l], acc[l]);
  float r = reduce_lanes(acc);
  for (int i = upper; i < size; i++) {
    float p = a[i] * b[i];
    r = r + p;
  }
  return r;
}

static void mm(const o_tensor *t, const float *x, float *out, int dim0, int dim1, int nthreads) {
  o_matmul(t->type, t->data, 0, x, out, dim0, dim1, nthreads, g_vector_api);
}

int o_argmax(const float *v, int n) {
  int best = 0;
  float bv = v[0];
  for (int i = 0; i < n; i++)
    if (v[i] > bv) {
      bv = v[i];
      best = i;
    }
  return best;
}

const float *o_forward(const o_model *m, o_state *s, int token, int position, int nthreads) {
  const int dim = m->dim;
  const float sqrt_dim = (float)sqrt((double)dim);
  /* Llama.kt:112-113 */
  for (int i = 0; i < dim; i++) s->x[i] = o_get(m->tok_embd.type, m->tok_embd.data, (int64_t)token * dim + i);
  for (int i = 0; i < dim; i++) s->x[i] = s->x[i] * sqrt_dim;

  for (int l = 0; l < m->n_layers; l++) {
    const o_layer *L = &m->layers[l];
    const int swa = m->is_swa[l];
    const int hs = head_size_of(m, l);
    const int qdim = m->n_heads * hs, kvdim = kv_dim_of(m, l), hidden = m->ff[l];
    const float *fr = swa ? s->cr_swa : s->cr_full, *fi = swa ? s->ci_swa : s->ci_full;
    /* Llama.kt:155-161 */
    o_rmsnorm(s->xb, s->x, L->attn_norm, dim, m->eps);
    mm(&L->wq, s->xb, s->q, qdim, dim, nthreads);
    for (int h = 0; h < m->n_heads; h++) rmsnorm_off(s->q + h * hs, s->q + h * hs, L->attn_q_norm, hs, m->eps);
    for (int h = 0; h < m->n_heads; h++) rope(s->q, h, hs, fr, fi, position);
    /* Llama.kt:170-196 */
    const int kv_layer = l < m->n_layer_kv_from_start ? l : m->n_layer_kv_from_start - (swa ? 2 : 1);
    const int nkv = m->n_kv_heads[l], kv_mul = m->n_heads / nkv;
    if (l < m->n_layer_kv_from_start) {
      mm(&L->wk, s->xb, s->k, kvdim, dim, nthreads);
      if (L->wv.data) mm(&L->wv, s->xb, s->v, kvdim, dim, nthreads);
      else memcpy(s->v, s->k, sizeof(float) * kvdim);
      for (int h = 0; h < nkv; h++) {
        rmsnorm_off(s->k + h * hs, s->k + h * hs, L->attn_k_norm, hs, m->eps);
        rmsnorm_noweight(s->v + h * hs, s->v + h * hs, hs, m->eps);
      }
      for (int h = 0; h < nkv; h++) rope(s->k, h, hs, fr, fi, position);
      memcpy(s->key_cache[kv_layer] + (size_t)position * kvdim, s->k, sizeof(float) * kvdim);
      memcpy(s->value_cache[kv_layer] + (size_t)position * kvdim, s->v, sizeof(float) * kvdim);
    }
    /* Llama.kt:198-218 */
    const int att_start = swa ? (position - m->sliding_window + 1 > 0 ? position - m->sliding_window + 1 : 0) : 0;
    const float *kc = s->key_cache[kv_layer], *vc = s->value_cache[kv_layer];
    for (int h = 0; h < m->n_heads; h++) {
      float *att = s->att + (size_t)h * m->ctx_len;
      for (int t = att_start; t <= position; t++)
        att[t] = array_dot(s->q + h * hs, kc + (size_t)t * kvdim + (h / kv_mul) * hs, hs);
      o_softmax(att + att_start, position - att_start + 1);
      float *xo = s->xbk + h * hs;
      for (int i = 0; i < hs; i++) xo[i] = 0.0f;
      for (int t = att_start; t <= position; t++) {
        const float *vv = vc + (size_t)t * kvdim + (h / kv_mul) * hs;
        float a = att[t];
        for (int i = 0; i < hs; i++) {
          float p = a * vv[i];
          xo[i] = p + xo[i];
        }
      }
    }
    /* Llama.kt:221-223 */
    mm(&L->wo, s->xbk, s->xb2, dim, qdim, nthreads);
    o_rmsnorm(s->xb2, s->xb2, L->post_attention_norm, dim, m->eps);
    for (int i = 0; i < dim; i++) s->x[i] = s->x[i] + s->xb2[i];
    /* Llama.kt:226-364 */
    o_rmsnorm(s->xb, s->x, L->ffn_norm, dim, m->eps);
    mm(&L->w1, s->xb, s->hb, hidden, dim, nthreads);
    mm(&L->w3, s->xb, s->hb2, hidden, dim, nthreads);
    for (int i = 0; i < hidden; i++) s->hb[i] = o_gelu(s->hb[i]);
    for (int i = 0; i < hidden; i++) s->hb[i] = s->hb[i] * s->hb2[i];
    mm(&L->w2, s->hb, s->xb, dim, hidden, nthreads);
    if (m->n_expert > 0) {
      o_rmsnorm(s->xb, s->xb, L->post_ffw_norm_1, dim, m->eps);
      o_moe_weights mw = {dim, m->n_expert, m->n_expert_used, m->expert_ff, m->eps,
                          L->gate_up_exps.type, L->down_exps.type, L->gate_inp.data, L->gate_inp_scale,
                          L->gate_up_exps.data, L->down_exps.data, L->down_exps_scale, L->pre_ffw_norm_2,
                          L->post_ffw_norm_2};
      int32_t idx[64];
      float prob[64];
      o_moe_token(&mw, s->x, s->moe_out, idx, prob, NULL, nthreads);
      for (int i = 0; i < dim; i++) s->xb[i] = s->xb[i] + s->moe_out[i];
    }
    o_rmsnorm(s->xb, s->xb, L->post_ffw_norm, dim, m->eps);
    for (int i = 0; i < dim; i++) s->x[i] = s->x[i] + s->xb[i];
    /* Llama.kt:393-397 */
    const float sc = m->layer_scale[l];
    if (sc != 1.0f)
      for (int i = 0; i < dim; i++) s->x[i] = s->x[i] * sc;
  }
  /* Llama.kt:401-406 */
  o_rmsnorm(s->x, s->x, m->output_norm, dim, m->eps);
  const o_tensor *wcls = m->output.data ? &m->output : &m->tok_embd;
  mm(wcls, s->x, s->logits, m->vocab, dim, nthreads);
  if (m->logit_softcap > 0) {
    const float cap = m->logit_softcap;
    for (int i = 0; i < m->vocab; i++) {
      float t = s->logits[i] / cap;
      s->logits[i] = cap * (float)tanh((double)t);
    }
  }
  return s->logits;
}
