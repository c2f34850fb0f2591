/*
 * g4_synth.c -- host-side quantizers that turn fp32 weights into GGUF block
 * streams (Q8_0, Q4_K, Q6_K, BF16, F32), for synthetic models and benchmark
 * inputs.  The reference only reads blocks (it has no quantizer), so these
 * produce blocks that its decoders (Q8_0FloatTensor.kt:21-28,
 * Q4_KFloatTensor.kt:23-84, Q6_KFloatTensor.kt:26-73, BF16FloatTensor.kt:20-24)
 * interpret as a close approximation of the input.
 *
 * Q8_0 follows ggml's rule (d = amax/127, q = round(x/d)); Q4_K and Q6_K use a
 * simple min/max fit per sub-block -- the quantizer's quality only matters for
 * realism, never for parity (parity is checked on whatever bytes it emits).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <string.h>

#define QK_K 256

static uint16_t f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t exp = (x >> 23) & 0xFFu;
  uint32_t man = x & 0x7FFFFFu;
  if (exp == 0xFF) return (uint16_t)(sign | 0x7C00u | (man ? 0x200u : 0));
  int e = (int)exp - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7C00u);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    man |= 0x800000u;
    int shift = 14 - e;
    uint32_t h = man >> shift;
    uint32_t rem = man & ((1u << shift) - 1), halfway = 1u << (shift - 1);
    if (rem > halfway || (rem == halfway && (h & 1))) h++;
    return (uint16_t)(sign | h);
  }
  uint32_t h = ((uint32_t)e << 10) | (man >> 13);
  uint32_t rem = man & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1))) h++;
  return (uint16_t)(sign | h);
}

static float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16, exp = (h >> 10) & 0x1F, man = h & 0x3FF, b;
  if (exp == 0) {
    if (man == 0) b = sign;
    else {
      int e = 113;
      while (!(man & 0x400)) { man <<= 1; e--; }
      b = sign | ((uint32_t)e << 23) | ((man & 0x3FF) << 13);
    }
  } else if (exp == 31) b = sign | 0x7F800000u | (man << 13);
  else b = sign | ((exp + 112) << 23) | (man << 13);
  float f;
  memcpy(&f, &b, 4);
  return f;
}

static void put16(uint8_t *p, uint16_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); }

/* ggml's roundf-based Q8_0 (gguf-py quants.Q8_0.quantize_blocks is bit-exact with it) */
static void q8_0_block(const float *x, uint8_t *o) {
  float amax = 0.f;
  for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(x[i]));
  float d = amax / 127.f, id = d != 0.f ? 1.f / d : 0.f;
  put16(o, f32_to_f16(d));
  for (int i = 0; i < 32; i++) o[2 + i] = (uint8_t)(int8_t)roundf(x[i] * id);
}

static void q4_k_block(const float *x, uint8_t *o) {
  float scale[8], mins[8];
  float max_scale = 0.f, max_min = 0.f;
  for (int s = 0; s < 8; s++) {
    float mn = x[32 * s], mx = x[32 * s];
    for (int i = 1; i < 32; i++) { mn = fminf(mn, x[32 * s + i]); mx = fmaxf(mx, x[32 * s + i]); }
    if (mn > 0.f) mn = 0.f;
    scale[s] = (mx - mn) / 15.f;
    mins[s] = -mn;
    max_scale = fmaxf(max_scale, scale[s]);
    max_min = fmaxf(max_min, mins[s]);
  }
  uint16_t dh = f32_to_f16(max_scale / 63.f), mh = f32_to_f16(max_min / 63.f);
  float d = f16_to_f32(dh), dmin = f16_to_f32(mh);
  int sc[8], m[8];
  for (int s = 0; s < 8; s++) {
    int a = d > 0.f ? (int)lrintf(scale[s] / d) : 0;
    int b = dmin > 0.f ? (int)lrintf(mins[s] / dmin) : 0;
    sc[s] = a < 0 ? 0 : a > 63 ? 63 : a;
    m[s] = b < 0 ? 0 : b > 63 ? 63 : b;
  }
  put16(o, dh);
  put16(o + 2, mh);
  uint8_t *s = o + 4;
  for (int j = 0; j < 4; j++) {
    s[j] = (uint8_t)(sc[j] | ((sc[j + 4] >> 4) << 6));
    s[j + 4] = (uint8_t)(m[j] | ((m[j + 4] >> 4) << 6));
    s[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((m[j + 4] & 0xF) << 4));
  }
  uint8_t *qs = o + 16;
  for (int g = 0; g < 4; g++) {
    for (int i = 0; i < 32; i++) {
      int q[2];
      for (int h = 0; h < 2; h++) {
        int sub = 2 * g + h;
        float ds = d * (float)sc[sub], dm = dmin * (float)m[sub];
        int v = ds > 0.f ? (int)lrintf((x[64 * g + 32 * h + i] + dm) / ds) : 0;
        q[h] = v < 0 ? 0 : v > 15 ? 15 : v;
      }
      qs[32 * g + i] = (uint8_t)(q[0] | (q[1] << 4));
    }
  }
}

static void q6_k_block(const float *x, uint8_t *o) {
  float scale[16], max_scale = 0.f;
  for (int s = 0; s < 16; s++) {
    float amax = 0.f;
    for (int i = 0; i < 16; i++) amax = fmaxf(amax, fabsf(x[16 * s + i]));
    scale[s] = amax / 31.f;
    max_scale = fmaxf(max_scale, scale[s]);
  }
  uint16_t dh = f32_to_f16(max_scale / 127.f);
  float d = f16_to_f32(dh);
  int8_t sc[16];
  for (int s = 0; s < 16; s++) {
    int a = d > 0.f ? (int)lrintf(scale[s] / d) : 0;
    sc[s] = (int8_t)(a > 127 ? 127 : a < -128 ? -128 : a);
  }
  memset(o, 0, 210);
  uint8_t *ql = o, *qh = o + 128;
  for (int w = 0; w < QK_K; w++) {
    int half = w / 128, rem = w % 128, sub32 = rem / 32, l = rem % 32;
    float ds = d * (float)sc[w / 16];
    int v = ds != 0.f ? (int)lrintf(x[w] / ds) : 0;
    v = v < -32 ? -32 : v > 31 ? 31 : v;
    int q6 = v + 32;
    uint8_t *qlp = ql + half * 64 + (sub32 & 1) * 32 + l;
    if (sub32 < 2) *qlp |= (uint8_t)(q6 & 0xF);
    else *qlp |= (uint8_t)((q6 & 0xF) << 4);
    qh[half * 32 + l] |= (uint8_t)(((q6 >> 4) & 3) << (2 * sub32));
  }
  memcpy(o + 192, sc, 16);
  put16(o + 208, dh);
}

static void bf16_elem(const float *x, uint8_t *o) {
  uint32_t b;
  memcpy(&b, x, 4);
  if ((b & 0x7F800000u) == 0x7F800000u && (b & 0x7FFFFFu)) b = (b | 0x400000u);  /* keep NaN */
  else b = b + 0x7FFFu + ((b >> 16) & 1u);                                        /* RNE */
  put16(o, (uint16_t)(b >> 16));
}

typedef struct {
  int type;
  const float *src;
  uint8_t *dst;
  int64_t b0, b1;
} qjob;

static int blk_elems(int t) { return t == 8 ? 32 : (t == 12 || t == 14) ? QK_K : 1; }
static int blk_bytes(int t) { return t == 8 ? 34 : t == 12 ? 144 : t == 14 ? 210 : t == 30 ? 2 : t == 0 ? 4 : 0; }

static void *qworker(void *p) {
  qjob *j = (qjob *)p;
  int be = blk_elems(j->type), bb = blk_bytes(j->type);
  for (int64_t b = j->b0; b < j->b1; b++) {
    const float *x = j->src + b * be;
    uint8_t *o = j->dst + b * bb;
    switch (j->type) {
      case 8: q8_0_block(x, o); break;
      case 12: q4_k_block(x, o); break;
      case 14: q6_k_block(x, o); break;
      case 30: bf16_elem(x, o); break;
      case 0: memcpy(o, x, 4); break;
    }
  }
  return NULL;
}

/* Quantize n elements (a multiple of the type's block size) into dst
 * (n / block_elems * block_bytes bytes).  Returns 0, or -1 for a bad type/size. */
int g4s_quantize(int type, const float *src, int64_t n, uint8_t *dst, int nthreads) {
  int be = blk_elems(type), bb = blk_bytes(type);
  if (bb == 0 || n % be) return -1;
  int64_t nb = n / be;
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 64) nthreads = 64;
  if (nb < 4096) nthreads = 1;
  qjob jobs[64];
  pthread_t th[64];
  for (int t = 0; t < nthreads; t++) jobs[t] = (qjob){type, src, dst, nb * t / nthreads, nb * (t + 1) / nthreads};
  for (int t = 1; t < nthreads; t++) pthread_create(&th[t], NULL, qworker, &jobs[t]);
  qworker(&jobs[0]);
  for (int t = 1; t < nthreads; t++) pthread_join(th[t], NULL);
  return 0;
}

int64_t g4s_nbytes(int type, int64_t n) {
  int be = blk_elems(type), bb = blk_bytes(type);
  if (bb == 0 || n % be) return -1;
  return n / be * bb;
}

/* ------------------------------------------------------------------ fast normals
 * Seeded N(0, std) float32 values for large synthetic models, generated by
 * all host threads: value i belongs to chunk i >> 20, and each chunk has its
 * own xoshiro256** stream seeded by splitmix64 from (seed, stream, chunk), so
 * the output depends only on (seed, stream, n, std), not on the thread count.
 * Normals by the Marsaglia polar method in double, rounded to float. */
#define G4S_CHUNK_SHIFT 20

static uint64_t splitmix64(uint64_t *s) {
  uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

static inline uint64_t rotl64(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

typedef struct {
  uint64_t s[4];
} xoshiro;

static inline uint64_t xoshiro_next(xoshiro *r) {
  const uint64_t out = rotl64(r->s[1] * 5, 7) * 9, t = r->s[1] << 17;
  r->s[2] ^= r->s[0];
  r->s[3] ^= r->s[1];
  r->s[1] ^= r->s[2];
  r->s[0] ^= r->s[3];
  r->s[2] ^= t;
  r->s[3] = rotl64(r->s[3], 45);
  return out;
}

static inline double unit_open(xoshiro *r) { /* uniform in (-1, 1) */
  return ((double)(xoshiro_next(r) >> 11) + 0.5) * (2.0 / 9007199254740992.0) - 1.0;
}

typedef struct {
  uint64_t seed, stream;
  float *out;
  int64_t n, c0, c1;
  double std;
} njob;

static void *nworker(void *p) {
  njob *j = (njob *)p;
  for (int64_t c = j->c0; c < j->c1; c++) {
    uint64_t sm = j->seed * 0xD1B54A32D192ED03ull ^ j->stream * 0x8CB92BA72F3D8DD7ull ^ (uint64_t)c;
    xoshiro r;
    for (int k = 0; k < 4; k++) r.s[k] = splitmix64(&sm);
    const int64_t a = c << G4S_CHUNK_SHIFT;
    const int64_t b = a + ((int64_t)1 << G4S_CHUNK_SHIFT) < j->n ? a + ((int64_t)1 << G4S_CHUNK_SHIFT) : j->n;
    for (int64_t i = a; i < b; i += 2) {
      double u, v, s;
      do {
        u = unit_open(&r);
        v = unit_open(&r);
        s = u * u + v * v;
      } while (s >= 1.0 || s == 0.0);
      const double f = sqrt(-2.0 * log(s) / s) * j->std;
      j->out[i] = (float)(u * f);
      if (i + 1 < b) j->out[i + 1] = (float)(v * f);
    }
  }
  return NULL;
}

int g4s_normal(uint64_t seed, uint64_t stream, float *out, int64_t n, double std, int nthreads) {
  if (!out || n < 0) return -1;
  const int64_t chunks = (n + ((int64_t)1 << G4S_CHUNK_SHIFT) - 1) >> G4S_CHUNK_SHIFT;
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 256) nthreads = 256;
  if (nthreads > chunks) nthreads = chunks > 0 ? (int)chunks : 1;
  pthread_t th[256];
  njob jobs[256];
  for (int t = 0; t < nthreads; t++) {
    jobs[t] = (njob){seed, stream, out, n, chunks * t / nthreads, chunks * (t + 1) / nthreads, std};
  }
  for (int t = 1; t < nthreads; t++) pthread_create(&th[t], NULL, nworker, &jobs[t]);
  nworker(&jobs[0]);
  for (int t = 1; t < nthreads; t++) pthread_join(th[t], NULL);
  return 0;
}
