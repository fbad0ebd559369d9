/* Host-only restatement of the synthetic CSR generators of the benchmark
 * configurations -- TEST INFRASTRUCTURE ONLY.
 *
 * The library's generators (prefree-public_b200/csrc/gen.cuh) define row r of
 * each config as a pure function of (seed, r), with integer arithmetic and
 * exactly rounded doubles. This file states the same definitions again in
 * plain C, independently of the library, so that:
 *   - bench.py's reference arm builds its inputs without loading the
 *     library it is compared against;
 *   - tests pin the library's host and device generators to a second,
 *     separately written implementation (bit-identical row_ptr, col, val, x).
 *
 * The reference has no generator: it reads SuiteSparse files and overwrites
 * values and x with i % 15 (include/common.h:126-133,
 * test/test_cdspmv.cpp:290-292). value_mode 1 is that convention. The
 * configurations are the five of the benchmark (uniform rows, 5-point
 * Laplacian, power-law rows, long rows, banded + uniform).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define POWERLAW_CAP 200000
#define BAND_HALF 4096
/* floor(0.7 * 2^53) */
#define BAND_P53 6305039478318694ULL

enum { ST_COL = 1, ST_VAL = 2, ST_X = 3, ST_LEN = 4, ST_BAND = 5, ST_NORMAL = 16 };

static uint64_t fmix(uint64_t z) {
  z ^= z >> 30;
  z *= 0xBF58476D1CE4E5B9ULL;
  z ^= z >> 27;
  z *= 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

/* keyed hash of (seed, stream, a, b) */
static uint64_t key4(uint64_t seed, uint64_t stream, uint64_t a, uint64_t b) {
  uint64_t h = fmix(seed * 0x9E3779B97F4A7C15ULL + stream);
  h = fmix(h ^ (a * 0xD1B54A32D192ED03ULL + 0x632BE59BD9B4E019ULL));
  return fmix(h ^ (b * 0x8CB92BA72F3D8DD7ULL + 0x2545F4914F6CDD1DULL));
}

/* floor(h * range / 2^64): an integer in [0, range) */
static int64_t below(uint64_t h, int64_t range) {
  return (int64_t)(((unsigned __int128)h * (uint64_t)range) >> 64);
}

static double pm1(uint64_t h) { return ldexp((double)(h >> 11), -52) - 1.0; }
static double unit(uint64_t h) { return ldexp((double)(h >> 11), -53); }

static int64_t side_of(int64_t m) {
  int64_t g = (int64_t)sqrt((double)m);
  while (g > 0 && g * g > m) --g;
  while ((g + 1) * (g + 1) <= m) ++g;
  return g;
}

typedef struct {
  int cfg, value_mode;
  uint64_t seed;
  int64_t m, n, k, side;
  uint64_t *thr; /* config 3: thr[l] = floor(2^64 (l - 0.5)^-1.1) */
  int64_t cap;
} gspec;

/* Defaults of the five configurations; 0 on success. */
int oracle_gen_resolve(int cfg, int64_t *m, int64_t *n, int64_t *k) {
  static const int64_t dm[6] = {0, 100000, 2048LL * 2048, 4000000, 50000, 1LL << 26};
  static const int64_t dk[6] = {0, 16, 5, POWERLAW_CAP, 2000, 32};
  if (cfg < 1 || cfg > 5) return 1;
  if (*m <= 0) *m = dm[cfg];
  if (*n <= 0) *n = *m;
  if (*k <= 0) *k = dk[cfg];
  if (cfg == 2) {
    const int64_t g = side_of(*m);
    if (g * g != *m || *n != *m) return 1;
  }
  return 0;
}

static int make(gspec *s, int cfg, int value_mode, uint64_t seed, int64_t m, int64_t n,
                int64_t k) {
  memset(s, 0, sizeof(*s));
  if (oracle_gen_resolve(cfg, &m, &n, &k)) return 1;
  s->cfg = cfg;
  s->value_mode = value_mode;
  s->seed = seed;
  s->m = m;
  s->n = n;
  s->k = k;
  s->side = cfg == 2 ? side_of(m) : 0;
  if (cfg == 3) {
    s->cap = k < n ? k : n;
    s->thr = (uint64_t *)malloc(sizeof(uint64_t) * (size_t)(s->cap + 1));
    if (!s->thr) return 1;
    s->thr[0] = s->thr[1] = ~0ULL;
    for (int64_t l = 2; l <= s->cap; ++l)
      s->thr[l] = (uint64_t)ldexp(pow((double)l - 0.5, -1.1), 64);
  }
  return 0;
}

static void drop(gspec *s) { free(s->thr); }

static int64_t length_of(const gspec *s, int64_t r) {
  if (s->cfg == 2) {
    const int64_t i = r / s->side, j = r % s->side;
    return 1 + (i > 0) + (i < s->side - 1) + (j > 0) + (j < s->side - 1);
  }
  if (s->cfg == 3) {
    /* the largest l in [1, cap] with h < thr[l] (thr decreases in l) */
    const uint64_t h = key4(s->seed, ST_LEN, (uint64_t)r, 0);
    int64_t lo = 1, hi = s->cap;
    while (lo < hi) {
      const int64_t mid = (lo + hi + 1) / 2;
      if (h < s->thr[mid]) lo = mid;
      else hi = mid - 1;
    }
    return lo;
  }
  return s->k;
}

static int cmp_i32(const void *a, const void *b) {
  const int32_t x = *(const int32_t *)a, y = *(const int32_t *)b;
  return (x > y) - (x < y);
}

/* columns of row r (len of them), sorted and distinct */
static void columns_of(const gspec *s, int64_t r, int64_t len, int32_t *c) {
  for (int64_t j = 0; j < len; ++j) {
    const uint64_t h = key4(s->seed, ST_COL, (uint64_t)r, (uint64_t)j);
    if (s->cfg == 5) {
      if ((key4(s->seed, ST_BAND, (uint64_t)r, (uint64_t)j) >> 11) < BAND_P53) {
        int64_t v = r - BAND_HALF + below(h, 2 * BAND_HALF + 1);
        v = v < 0 ? 0 : (v > s->n - 1 ? s->n - 1 : v);
        c[j] = (int32_t)v;
      } else {
        c[j] = (int32_t)below(h, s->n);
      }
    } else {
      c[j] = (int32_t)below(h, s->n - len + 1);
    }
  }
  qsort(c, (size_t)len, sizeof(int32_t), cmp_i32);
  if (s->cfg == 5) {
    /* push equal neighbours apart upwards, then pull back under n */
    for (int64_t j = 1; j < len; ++j)
      if (c[j] <= c[j - 1]) c[j] = c[j - 1] + 1;
    if (len > 0 && c[len - 1] > s->n - 1) c[len - 1] = (int32_t)(s->n - 1);
    for (int64_t j = len - 2; j >= 0; --j)
      if (c[j] >= c[j + 1]) c[j] = c[j + 1] - 1;
  } else {
    /* sorted draws d_0 <= d_1 <= ... become d_j + j: strictly increasing */
    for (int64_t j = 0; j < len; ++j) c[j] += (int32_t)j;
  }
}

static double value_of(const gspec *s, int64_t r, int64_t j, int64_t g, double lap) {
  if (s->value_mode == 1) return (double)(g % 15);
  if (s->cfg == 2) return lap;
  if (s->cfg == 4) {
    /* Irwin-Hall(12) - 6, summed in this order */
    double t = 0.0;
    for (uint64_t q = 0; q < 12; ++q)
      t += unit(key4(s->seed, ST_NORMAL + q, (uint64_t)r, (uint64_t)j));
    return t - 6.0;
  }
  return pm1(key4(s->seed, ST_VAL, (uint64_t)r, (uint64_t)j));
}

static int64_t count_rows(const gspec *s, int64_t r0, int64_t r1) {
  if (s->cfg == 1 || s->cfg == 4 || s->cfg == 5) return (r1 - r0) * s->k;
  int64_t t = 0;
  for (int64_t r = r0; r < r1; ++r) t += length_of(s, r);
  return t;
}

/* Non-zeros of rows [r0, r1); -1 on a bad spec or range. */
int64_t oracle_gen_count(int cfg, int value_mode, uint64_t seed, int64_t m, int64_t n, int64_t k,
                         int64_t r0, int64_t r1) {
  gspec s;
  if (make(&s, cfg, value_mode, seed, m, n, k)) return -1;
  int64_t z = -1;
  if (0 <= r0 && r0 <= r1 && r1 <= s.m) z = count_rows(&s, r0, r1);
  drop(&s);
  return z;
}

/* Rows [r0, r1): row_ptr (r1 - r0 + 1 entries from 0), col, val (fp64).
 * 0 on success. */
int oracle_gen_rows(int cfg, int value_mode, uint64_t seed, int64_t m, int64_t n, int64_t k,
                    int64_t r0, int64_t r1, int64_t *row_ptr, int32_t *col, double *val) {
  gspec s;
  if (make(&s, cfg, value_mode, seed, m, n, k)) return 1;
  if (!(0 <= r0 && r0 <= r1 && r1 <= s.m)) {
    drop(&s);
    return 1;
  }
  const int64_t g0 = s.value_mode == 1 ? count_rows(&s, 0, r0) : 0;
  int64_t off = 0;
  row_ptr[0] = 0;
  for (int64_t r = r0; r < r1; ++r) {
    const int64_t len = length_of(&s, r);
    if (s.cfg == 2) {
      /* neighbours in column order: up, left, centre, right, down */
      const int64_t G = s.side, i = r / G, j = r % G;
      const int64_t nb[5] = {i > 0 ? r - G : -1, j > 0 ? r - 1 : -1, r,
                             j < G - 1 ? r + 1 : -1, i < G - 1 ? r + G : -1};
      int64_t q = off;
      for (int e = 0; e < 5; ++e) {
        if (nb[e] < 0) continue;
        col[q] = (int32_t)nb[e];
        val[q] = value_of(&s, r, q - off, g0 + q, e == 2 ? 4.0 : -1.0);
        ++q;
      }
    } else {
      columns_of(&s, r, len, col + off);
      for (int64_t j = 0; j < len; ++j) val[off + j] = value_of(&s, r, j, g0 + off + j, 0.0);
    }
    off += len;
    row_ptr[r - r0 + 1] = off;
  }
  drop(&s);
  return 0;
}

/* x[c0 .. c1). 0 on success. */
int oracle_gen_x(int cfg, int value_mode, uint64_t seed, int64_t m, int64_t n, int64_t k,
                 int64_t c0, int64_t c1, double *x) {
  if (oracle_gen_resolve(cfg, &m, &n, &k) || !(0 <= c0 && c0 <= c1 && c1 <= n)) return 1;
  for (int64_t c = c0; c < c1; ++c)
    x[c - c0] = value_mode == 1 ? (double)(c % 15) : pm1(key4(seed, ST_X, (uint64_t)c, 0));
  return 0;
}
