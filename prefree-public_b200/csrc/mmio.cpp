// Matrix Market -> CSR reader: the harness input path of the reference
// (mmio_allinone, utilities/mmio.cpp:1547-1713), rebuilt as a parallel parser.
//
// Same results as the reference for coordinate files:
//   * banner "%%MatrixMarket matrix coordinate <type> <symmetry>", tokens
//     case-insensitive (mm_read_banner, mmio.cpp:246-330);
//   * comment lines (leading '%') skipped before the "M N NZ" size line
//     (mm_read_mtx_crd_size, mmio.cpp:416-447);
//   * values: real as parsed (strtod, the conversion scanf's %lg uses),
//     integer converted to double, pattern = 1.0, complex = real part
//     (mmio.cpp:1602-1636);
//   * 1-based -> 0-based (:1629-1630);
//   * symmetric and hermitian files mirror every off-diagonal entry into the
//     column's row (:1641-1648); skew-symmetric files are NOT mirrored (the
//     reference tests only mm_is_symmetric / mm_is_hermitian);
//   * CSR by counting sort in file order: entry k lands in row i after every
//     earlier entry of row i, and its mirror lands in row j right after that
//     (:1650-1695). Column order inside a row is therefore file order.
// Differences: int64 row_ptr/nnz; the file is read, the entry lines parsed
// and the CSR built by several threads (the CSR build stays in file order:
// each thread owns a range of rows and places its entries in file order);
// dense "array" files and malformed input return an error instead of reading
// garbage.
#include <algorithm>
#include <cctype>
#include <cerrno>
#include <charconv>
#include <climits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include "../../include/prefree_b200.h"

namespace pf {
void set_error(const char *fmt, ...);
}

namespace {

struct Entries {
  std::unique_ptr<int32_t[]> ri, ci;  // left uninitialised: every slot is written
  std::unique_ptr<double[]> v;
};

// strtoll on a token, without copying it: optional sign, then base-10 digits
// up to the first other character; saturates like strtoll. False when no
// digit follows the sign.
inline bool parse_ll(const char *s, const char *e, long long *out) {
  bool neg = false;
  if (s < e && (*s == '+' || *s == '-')) {
    neg = *s == '-';
    ++s;
  }
  if (s >= e || *s < '0' || *s > '9') return false;
  unsigned long long x = 0;
  bool ovf = false;
  for (; s < e && *s >= '0' && *s <= '9'; ++s) {
    const unsigned d = (unsigned)(*s - '0');
    if (x > (ULLONG_MAX - d) / 10) ovf = true;
    else x = x * 10 + d;
  }
  if (neg) *out = (ovf || x > (unsigned long long)LLONG_MAX + 1) ? LLONG_MIN : (long long)(0 - x);
  else *out = (ovf || x > (unsigned long long)LLONG_MAX) ? LLONG_MAX : (long long)x;
  return true;
}

// strtod on a token: std::from_chars (correctly rounded, as glibc's strtod)
// when it takes the whole token and gives a number; anything else (a leading
// '+', hex, out of range, NaN, trailing characters) goes through strtod on a
// copy, so the value is always strtod's
inline bool parse_double(const char *tb, size_t tl, double *out) {
  double v;
  const auto r = std::from_chars(tb, tb + tl, v);
  if (r.ec == std::errc() && r.ptr == tb + tl && !std::isnan(v)) {
    *out = v;
    return true;
  }
  char buf[128];
  if (tl >= sizeof(buf)) return false;
  std::memcpy(buf, tb, tl);
  buf[tl] = 0;
  char *e = nullptr;
  *out = std::strtod(buf, &e);
  return e != buf;
}

// the C locale's isspace, inline (the parse calls it for every character)
inline bool is_space(char c) {
  return c == ' ' || c == '\t' || c == '\n' || c == '\v' || c == '\f' || c == '\r';
}

inline const char *skip_ws(const char *p, const char *end) {
  while (p < end && (*p == ' ' || *p == '\t' || *p == '\r')) ++p;
  return p;
}

// Parse one entry line [p, eol). Returns false on malformed input.
inline bool parse_entry(const char *p, const char *eol, int nv, bool is_int,
                        int64_t *i, int64_t *j, double *val) {
  const char *q = p;
  auto next_token = [&](const char **tb, size_t *tl) -> bool {
    q = skip_ws(q, eol);
    if (q >= eol) return false;
    const char *s = q;
    while (q < eol && !is_space(*q)) ++q;
    *tb = s;
    *tl = (size_t)(q - s);
    return true;
  };
  const char *tb;
  size_t tl;
  constexpr size_t kMaxToken = 127;  // longer tokens are malformed
  for (int f = 0; f < 2; ++f) {
    long long x;
    if (!next_token(&tb, &tl) || tl > kMaxToken || !parse_ll(tb, tb + tl, &x)) return false;
    (f == 0 ? *i : *j) = x;
  }
  if (nv == 0) {
    *val = 1.0;
    return true;
  }
  if (!next_token(&tb, &tl) || tl > kMaxToken) return false;
  if (is_int) {
    long long x;
    if (!parse_ll(tb, tb + tl, &x)) return false;
    *val = (double)(int)x;
    return true;
  }
  return parse_double(tb, tl, val);  // a complex file's imaginary part is ignored
}

// Host threads for a pass over `bytes` bytes (one below 64 MB).
unsigned host_threads(size_t bytes) {
  if (bytes < ((size_t)64 << 20)) return 1;
  return std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
}

// Runs fn(k) for k in [0, nthr) on nthr threads (inline when nthr is 1).
template <typename F>
void run_threads(unsigned nthr, F &&fn) {
  if (nthr <= 1) {
    fn(0u);
    return;
  }
  std::vector<std::thread> th;
  for (unsigned k = 0; k < nthr; ++k) th.emplace_back(fn, k);
  for (auto &t : th) t.join();
}

// Reads n bytes at file offset off into dst, in parallel pieces; false on a
// short read or an error (errno says which).
bool pread_all(int fd, char *dst, size_t n, size_t off) {
  const unsigned nthr = host_threads(n);
  std::vector<int> ok(nthr, 1);
  run_threads(nthr, [&](unsigned k) {
    size_t a = n * k / nthr;
    const size_t e = n * (k + 1) / nthr;
    while (a < e) {
      const ssize_t r = ::pread(fd, dst + a, e - a, (off_t)(off + a));
      if (r <= 0) {
        if (r < 0 && errno == EINTR) continue;
        ok[k] = 0;
        return;
      }
      a += (size_t)r;
    }
  });
  return std::all_of(ok.begin(), ok.end(), [](int v) { return v != 0; });
}

// Reads a whole file into a NUL-terminated buffer, in parallel pieces.
// 0: done; 1: the file cannot be opened; 2: it cannot be read (errno says why).
int read_file(const char *path, std::unique_ptr<char[]> *buf, size_t *size) {
  const int fd = ::open(path, O_RDONLY);
  if (fd < 0) return 1;
  struct stat st;
  if (::fstat(fd, &st) != 0 || st.st_size < 0) {
    ::close(fd);
    return 2;
  }
  const size_t n = (size_t)st.st_size;
  buf->reset(new (std::nothrow) char[n + 1]);
  if (!*buf) {
    ::close(fd);
    errno = ENOMEM;
    return 2;
  }
  char *b = buf->get();
  b[n] = 0;
  const bool ok = pread_all(fd, b, n, 0);
  ::close(fd);
  *size = n;
  return ok ? 0 : 2;
}

// Equal-nnz row split (see the header).
template <typename IT>
pf_status shard_bounds(const IT *rp, int64_t m, int parts, int64_t *b) {
  if (!rp || !b || m < 0 || parts < 1) {
    pf::set_error("pf_shard_bounds: bad arguments");
    return PF_ERR_INVALID;
  }
  const int64_t base = (int64_t)rp[0];
  const int64_t z = (int64_t)rp[m] - base;
  b[0] = 0;
  for (int k = 1; k < parts; ++k) {
    const int64_t target = base + (int64_t)((__int128)z * k / parts);
    int64_t lo = 0, hi = m;  // first r with rp[r] >= target
    while (lo < hi) {
      const int64_t mid = (lo + hi) / 2;
      if ((int64_t)rp[mid] >= target) hi = mid;
      else lo = mid + 1;
    }
    b[k] = std::max(lo, b[k - 1]);
  }
  b[parts] = m;
  return PF_OK;
}

}  // namespace

namespace pf {
// Page-locked host memory for the loader's output arrays (defined in
// spmv_api.cu, which talks to the CUDA runtime): null on failure; and the
// free of an array this library returned, pinned or not.
void *pinned_alloc(size_t bytes);
bool pinned_free(void *p);  // false: p was not page-locked memory
}  // namespace pf

namespace {
// the loader's output arrays: heap (malloc) or page-locked
void *out_alloc(size_t bytes, bool pinned, bool zero) {
  void *p = pinned ? pf::pinned_alloc(bytes) : std::malloc(bytes);
  if (p && zero) std::memset(p, 0, bytes);
  return p;
}
void out_free(void *p, bool pinned) {
  if (!p) return;
  if (pinned) pf::pinned_free(p);
  else std::free(p);
}
}  // namespace

extern "C" {

void pf_free(void *p) {
  if (p && !pf::pinned_free(p)) std::free(p);
}

static pf_status mmio_read_impl(const char *path, int64_t *m_out, int64_t *n_out,
                                int64_t *nnz_out, int *sym_out, int64_t **row_ptr_out,
                                int32_t **col_out, double **val_out, bool pinned) {
  if (!path || !m_out || !n_out || !nnz_out || !sym_out || !row_ptr_out || !col_out ||
      !val_out) {
    pf::set_error("pf_mmio_read: null argument");
    return PF_ERR_INVALID;
  }
  std::unique_ptr<char[]> text;
  size_t text_size = 0;
  const int rf = read_file(path, &text, &text_size);
  if (rf != 0) {
    pf::set_error("pf_mmio_read: cannot %s %s: %s", rf == 1 ? "open" : "read", path,
                  std::strerror(errno));
    return PF_ERR_IO;
  }
  const char *p = text.get();
  const char *end = p + text_size;
  auto line_end = [&](const char *s) {
    const char *e = (const char *)std::memchr(s, '\n', (size_t)(end - s));
    return e ? e : end;
  };

  // banner
  const char *eol = line_end(p);
  std::string banner(p, eol);
  char t[5][64];
  if (std::sscanf(banner.c_str(), "%63s %63s %63s %63s %63s", t[0], t[1], t[2], t[3], t[4]) != 5) {
    pf::set_error("pf_mmio_read: bad banner");
    return PF_ERR_FORMAT;
  }
  for (int k = 1; k < 5; ++k)
    for (char *c = t[k]; *c; ++c) *c = (char)std::tolower((unsigned char)*c);
  if (std::strncmp(t[0], "%%MatrixMarket", 14) != 0 || std::strcmp(t[1], "matrix") != 0) {
    pf::set_error("pf_mmio_read: not a Matrix Market matrix file");
    return PF_ERR_FORMAT;
  }
  if (std::strcmp(t[2], "coordinate") != 0) {
    pf::set_error("pf_mmio_read: only coordinate (sparse) files are supported");
    return PF_ERR_FORMAT;
  }
  int nv;
  bool is_int = false;
  if (!std::strcmp(t[3], "real")) nv = 1;
  else if (!std::strcmp(t[3], "integer")) { nv = 1; is_int = true; }
  else if (!std::strcmp(t[3], "complex")) nv = 2;
  else if (!std::strcmp(t[3], "pattern")) nv = 0;
  else {
    pf::set_error("pf_mmio_read: unknown data type %s", t[3]);
    return PF_ERR_FORMAT;
  }
  const bool sym = !std::strcmp(t[4], "symmetric") || !std::strcmp(t[4], "hermitian");

  // comments, then the size line
  p = eol < end ? eol + 1 : end;
  long long M = 0, N = 0, NZ = 0;
  while (p < end) {
    eol = line_end(p);
    const char *q = skip_ws(p, eol);
    if (q < eol && *q == '%') { p = eol + 1; continue; }
    if (q >= eol) { p = eol + 1; continue; }  // blank line
    std::string sl(q, eol);
    if (std::sscanf(sl.c_str(), "%lld %lld %lld", &M, &N, &NZ) != 3) {
      pf::set_error("pf_mmio_read: bad size line");
      return PF_ERR_FORMAT;
    }
    p = eol < end ? eol + 1 : end;
    break;
  }
  if (M <= 0 || N <= 0 || NZ < 0 || M > INT32_MAX || N > INT32_MAX) {
    pf::set_error("pf_mmio_read: bad sizes M=%lld N=%lld NZ=%lld", M, N, NZ);
    return PF_ERR_FORMAT;
  }

  // split the entry region into line-aligned chunks, count entries per chunk
  unsigned nthr = std::max(1u, std::min(64u, std::thread::hardware_concurrency()));
  if ((size_t)(end - p) < (1u << 20)) nthr = 1;
  std::vector<const char *> cut(nthr + 1);
  cut[0] = p;
  for (unsigned k = 1; k < nthr; ++k) {
    const char *c = p + (size_t)(end - p) * k / nthr;
    if (c < cut[k - 1]) c = cut[k - 1];
    const char *e = (const char *)std::memchr(c, '\n', (size_t)(end - c));
    cut[k] = e ? e + 1 : end;
  }
  cut[nthr] = end;
  auto is_entry_line = [](const char *s, const char *e) {
    s = skip_ws(s, e);
    return s < e && *s != '%';
  };
  std::vector<int64_t> cnt(nthr + 1, 0);
  {
    std::vector<std::thread> th;
    for (unsigned k = 0; k < nthr; ++k)
      th.emplace_back([&, k]() {
        int64_t c = 0;
        for (const char *s = cut[k]; s < cut[k + 1];) {
          const char *e = (const char *)std::memchr(s, '\n', (size_t)(cut[k + 1] - s));
          if (!e) e = cut[k + 1];
          if (is_entry_line(s, e)) ++c;
          s = e + 1;
        }
        cnt[k + 1] = c;
      });
    for (auto &x : th) x.join();
  }
  for (unsigned k = 0; k < nthr; ++k) cnt[k + 1] += cnt[k];
  if (cnt[nthr] < NZ) {
    pf::set_error("pf_mmio_read: file has %lld entries, header says %lld",
                  (long long)cnt[nthr], NZ);
    return PF_ERR_FORMAT;
  }
  Entries E;
  E.ri.reset(new (std::nothrow) int32_t[(size_t)std::max<long long>(NZ, 1)]);
  E.ci.reset(new (std::nothrow) int32_t[(size_t)std::max<long long>(NZ, 1)]);
  E.v.reset(new (std::nothrow) double[(size_t)std::max<long long>(NZ, 1)]);
  if (!E.ri || !E.ci || !E.v) {
    pf::set_error("pf_mmio_read: out of host memory");
    return PF_ERR_INVALID;
  }
  std::vector<int> bad(nthr, 0);
  {
    std::vector<std::thread> th;
    for (unsigned k = 0; k < nthr; ++k)
      th.emplace_back([&, k]() {
        int64_t o = cnt[k];
        for (const char *s = cut[k]; s < cut[k + 1] && o < NZ;) {
          const char *e = (const char *)std::memchr(s, '\n', (size_t)(cut[k + 1] - s));
          if (!e) e = cut[k + 1];
          if (is_entry_line(s, e)) {
            int64_t i, j;
            double v;
            if (!parse_entry(s, e, nv, is_int, &i, &j, &v) || i < 1 || i > M || j < 1 ||
                j > N) {
              bad[k] = 1;
              return;
            }
            E.ri[(size_t)o] = (int32_t)(i - 1);
            E.ci[(size_t)o] = (int32_t)(j - 1);
            E.v[(size_t)o] = v;
            ++o;
          }
          s = e + 1;
        }
      });
    for (auto &x : th) x.join();
  }
  for (unsigned k = 0; k < nthr; ++k)
    if (bad[k]) {
      pf::set_error("pf_mmio_read: malformed entry or index out of range");
      return PF_ERR_FORMAT;
    }
  if (sym && M != N) {
    pf::set_error("pf_mmio_read: symmetric file with M != N");
    return PF_ERR_FORMAT;
  }
  text.reset();

  // counting sort in file order: row counts (threads add atomically), then
  // each thread owns an equal-nnz range of rows and walks all entries in file
  // order, placing the ones (and the mirrors) that land in its rows, so every
  // row receives its entries in the same order as a single pass would give
  int64_t *rp = (int64_t *)out_alloc(sizeof(int64_t) * ((size_t)M + 1), pinned, true);
  if (!rp) {
    pf::set_error("pf_mmio_read: out of host memory%s", pinned ? " (page-locked)" : "");
    return PF_ERR_INVALID;
  }
  unsigned ncsr = std::max(1u, std::min(64u, std::thread::hardware_concurrency()));
  if (NZ < (1 << 20)) ncsr = 1;
  auto parallel = [&](auto &&fn) { run_threads(ncsr, fn); };
  parallel([&](unsigned k) {
    const int64_t a = NZ * (int64_t)k / ncsr, b = NZ * (int64_t)(k + 1) / ncsr;
    for (int64_t q = a; q < b; ++q) {
      const int32_t i = E.ri[(size_t)q], j = E.ci[(size_t)q];
      __atomic_fetch_add(&rp[i], 1, __ATOMIC_RELAXED);
      if (sym && i != j) __atomic_fetch_add(&rp[j], 1, __ATOMIC_RELAXED);
    }
  });
  int64_t run = 0;
  for (int64_t r = 0; r <= M; ++r) {
    const int64_t c = rp[r];
    rp[r] = run;
    run += c;
  }
  const int64_t nnz = run;
  int32_t *col = (int32_t *)out_alloc(sizeof(int32_t) * (size_t)std::max<int64_t>(nnz, 1), pinned,
                                      false);
  double *val = (double *)out_alloc(sizeof(double) * (size_t)std::max<int64_t>(nnz, 1), pinned,
                                    false);
  if (!col || !val) {
    out_free(rp, pinned);
    out_free(col, pinned);
    out_free(val, pinned);
    pf::set_error("pf_mmio_read: out of host memory%s", pinned ? " (page-locked)" : "");
    return PF_ERR_INVALID;
  }
  // row ranges of equal nnz (thread k owns rows [rb[k], rb[k + 1]))
  std::vector<int64_t> rb(ncsr + 1);
  shard_bounds(rp, M, (int)ncsr, rb.data());
  parallel([&](unsigned k) {
    const int32_t r0 = (int32_t)rb[k], r1 = (int32_t)rb[k + 1];
    if (r0 >= r1) return;
    std::vector<int64_t> cur(rp + r0, rp + r1);  // next slot of each owned row
    for (int64_t q = 0; q < NZ; ++q) {
      const int32_t i = E.ri[(size_t)q];
      const bool mine = i >= r0 && i < r1;
      if (!sym && !mine) continue;
      const int32_t j = E.ci[(size_t)q];
      if (mine) {
        const int64_t o = cur[(size_t)(i - r0)]++;
        col[o] = j;
        val[o] = E.v[(size_t)q];
      }
      if (sym && i != j && j >= r0 && j < r1) {
        const int64_t o = cur[(size_t)(j - r0)]++;
        col[o] = i;
        val[o] = E.v[(size_t)q];
      }
    }
  });
  *m_out = M;
  *n_out = N;
  *nnz_out = nnz;
  *sym_out = sym ? 1 : 0;
  *row_ptr_out = rp;
  *col_out = col;
  *val_out = val;
  return PF_OK;
}

// ---- binary CSR cache ---------------------------------------------------------
// File: a 64-byte header {magic "PFCSR001", m, n, nnz, is_symmetric, source
// size, source mtime in ns, 0}, then row_ptr (int64, m+1), col (int32, nnz),
// val (double, nnz), all little-endian as in memory.

struct CsrHeader {
  char magic[8];
  int64_t m, n, nnz, sym, src_size, src_mtime_ns, pad;
};
static const char kCsrMagic[8] = {'P', 'F', 'C', 'S', 'R', '0', '0', '1'};

static bool file_stamp(const char *path, int64_t *size, int64_t *mtime_ns) {
  struct stat st;
  if (stat(path, &st) != 0) return false;
  *size = (int64_t)st.st_size;
  *mtime_ns = (int64_t)st.st_mtim.tv_sec * 1000000000LL + (int64_t)st.st_mtim.tv_nsec;
  return true;
}

static pf_status csr_write(const char *path, int64_t m, int64_t n, int64_t nnz, int sym,
                           const int64_t *rp, const int32_t *col, const double *val,
                           int64_t src_size, int64_t src_mtime_ns) {
  if (!path || m < 0 || n < 0 || nnz < 0 || !rp || (nnz > 0 && (!col || !val))) {
    pf::set_error("pf_csr_write: bad argument");
    return PF_ERR_INVALID;
  }
  const std::string tmp = std::string(path) + ".tmp";
  FILE *f = std::fopen(tmp.c_str(), "wb");
  if (!f) {
    pf::set_error("pf_csr_write: cannot create %s: %s", tmp.c_str(), std::strerror(errno));
    return PF_ERR_IO;
  }
  CsrHeader hd;
  std::memcpy(hd.magic, kCsrMagic, 8);
  hd.m = m;
  hd.n = n;
  hd.nnz = nnz;
  hd.sym = sym;
  hd.src_size = src_size;
  hd.src_mtime_ns = src_mtime_ns;
  hd.pad = 0;
  bool ok = std::fwrite(&hd, sizeof(hd), 1, f) == 1 &&
            std::fwrite(rp, sizeof(int64_t), (size_t)m + 1, f) == (size_t)m + 1 &&
            (nnz == 0 || (std::fwrite(col, sizeof(int32_t), (size_t)nnz, f) == (size_t)nnz &&
                          std::fwrite(val, sizeof(double), (size_t)nnz, f) == (size_t)nnz));
  ok = (std::fclose(f) == 0) && ok;
  if (!ok || std::rename(tmp.c_str(), path) != 0) {
    std::remove(tmp.c_str());
    pf::set_error("pf_csr_write: write to %s failed", path);
    return PF_ERR_IO;
  }
  return PF_OK;
}

// Reads a cache file; with want_size >= 0 the recorded source stamp must
// match (want_size, want_mtime), else PF_ERR_FORMAT.
static pf_status csr_read(const char *path, int64_t want_size, int64_t want_mtime, int64_t *m_out,
                          int64_t *n_out, int64_t *nnz_out, int *sym_out, int64_t **rp_out,
                          int32_t **col_out, double **val_out, bool pinned) {
  const int fd = ::open(path, O_RDONLY);
  if (fd < 0) {
    pf::set_error("pf_csr_read: cannot open %s: %s", path, std::strerror(errno));
    return PF_ERR_IO;
  }
  CsrHeader hd;
  int64_t fsize = -1, fmt = 0;
  file_stamp(path, &fsize, &fmt);
  if (!pread_all(fd, (char *)&hd, sizeof(hd), 0) || std::memcmp(hd.magic, kCsrMagic, 8) != 0 ||
      hd.m < 0 || hd.n < 0 || hd.nnz < 0 || hd.m >= ((int64_t)1 << 40) ||
      hd.nnz >= ((int64_t)1 << 40) ||
      fsize != (int64_t)sizeof(hd) + 8 * (hd.m + 1) + 12 * hd.nnz ||
      (want_size >= 0 && (hd.src_size != want_size || hd.src_mtime_ns != want_mtime))) {
    ::close(fd);
    pf::set_error("pf_csr_read: %s is not a matching CSR cache file", path);
    return PF_ERR_FORMAT;
  }
  int64_t *rp = (int64_t *)out_alloc(sizeof(int64_t) * (size_t)(hd.m + 1), pinned, false);
  int32_t *col =
      (int32_t *)out_alloc(sizeof(int32_t) * (size_t)std::max<int64_t>(hd.nnz, 1), pinned, false);
  double *val =
      (double *)out_alloc(sizeof(double) * (size_t)std::max<int64_t>(hd.nnz, 1), pinned, false);
  const size_t rp_bytes = sizeof(int64_t) * (size_t)(hd.m + 1);
  const size_t col_bytes = sizeof(int32_t) * (size_t)hd.nnz;
  bool ok = rp && col && val && pread_all(fd, (char *)rp, rp_bytes, sizeof(hd)) &&
            (hd.nnz == 0 ||
             (pread_all(fd, (char *)col, col_bytes, sizeof(hd) + rp_bytes) &&
              pread_all(fd, (char *)val, sizeof(double) * (size_t)hd.nnz,
                        sizeof(hd) + rp_bytes + col_bytes)));
  ::close(fd);
  // the CSR must be consistent before anyone indexes with it
  if (ok) ok = rp[0] == 0 && rp[hd.m] == hd.nnz;
  if (ok) {
    const unsigned nthr = host_threads(col_bytes + rp_bytes);
    std::vector<int> good(nthr, 1);
    run_threads(nthr, [&](unsigned t) {
      const int64_t r0 = hd.m * (int64_t)t / nthr, r1 = hd.m * (int64_t)(t + 1) / nthr;
      for (int64_t r = r0; r < r1; ++r)
        if (rp[r] > rp[r + 1]) {
          good[t] = 0;
          return;
        }
      const int64_t k0 = hd.nnz * (int64_t)t / nthr, k1 = hd.nnz * (int64_t)(t + 1) / nthr;
      for (int64_t k = k0; k < k1; ++k)
        if (col[k] < 0 || (int64_t)col[k] >= hd.n) {
          good[t] = 0;
          return;
        }
    });
    ok = std::all_of(good.begin(), good.end(), [](int v) { return v != 0; });
  }
  if (!ok) {
    out_free(rp, pinned);
    out_free(col, pinned);
    out_free(val, pinned);
    pf::set_error("pf_csr_read: %s is truncated or inconsistent", path);
    return PF_ERR_FORMAT;
  }
  *m_out = hd.m;
  *n_out = hd.n;
  *nnz_out = hd.nnz;
  *sym_out = (int)hd.sym;
  *rp_out = rp;
  *col_out = col;
  *val_out = val;
  return PF_OK;
}

pf_status pf_csr_write(const char *path, int64_t m, int64_t n, int64_t nnz, int is_symmetric,
                       const int64_t *row_ptr, const int32_t *col_idx, const double *val) {
  return csr_write(path, m, n, nnz, is_symmetric, row_ptr, col_idx, val, -1, 0);
}

pf_status pf_csr_read(const char *path, int64_t *m, int64_t *n, int64_t *nnz, int *is_symmetric,
                      int64_t **row_ptr, int32_t **col_idx, double **val) {
  if (!path || !m || !n || !nnz || !is_symmetric || !row_ptr || !col_idx || !val) {
    pf::set_error("pf_csr_read: null argument");
    return PF_ERR_INVALID;
  }
  return csr_read(path, -1, 0, m, n, nnz, is_symmetric, row_ptr, col_idx, val, false);
}

static pf_status mmio_read_cached_impl(const char *mtx_path, const char *cache_path, int64_t *m,
                                       int64_t *n, int64_t *nnz, int *is_symmetric,
                                       int64_t **row_ptr, int32_t **col_idx, double **val,
                                       int *from_cache, bool pinned) {
  if (!mtx_path || !cache_path || !m || !n || !nnz || !is_symmetric || !row_ptr || !col_idx ||
      !val) {
    pf::set_error("pf_mmio_read_cached: null argument");
    return PF_ERR_INVALID;
  }
  int64_t sz = 0, mt = 0;
  if (!file_stamp(mtx_path, &sz, &mt)) {
    pf::set_error("pf_mmio_read_cached: cannot stat %s: %s", mtx_path, std::strerror(errno));
    return PF_ERR_IO;
  }
  if (from_cache) *from_cache = 0;
  if (csr_read(cache_path, sz, mt, m, n, nnz, is_symmetric, row_ptr, col_idx, val, pinned) ==
      PF_OK) {
    if (from_cache) *from_cache = 1;
    return PF_OK;
  }
  pf_status st = mmio_read_impl(mtx_path, m, n, nnz, is_symmetric, row_ptr, col_idx, val, pinned);
  if (st != PF_OK) return st;
  // best effort: a cache that cannot be written only costs the next parse
  csr_write(cache_path, *m, *n, *nnz, *is_symmetric, *row_ptr, *col_idx, *val, sz, mt);
  return PF_OK;
}

pf_status pf_mmio_read(const char *path, int64_t *m, int64_t *n, int64_t *nnz, int *is_symmetric,
                       int64_t **row_ptr, int32_t **col_idx, double **val) {
  return mmio_read_impl(path, m, n, nnz, is_symmetric, row_ptr, col_idx, val, false);
}

pf_status pf_mmio_read_pinned(const char *path, int64_t *m, int64_t *n, int64_t *nnz,
                              int *is_symmetric, int64_t **row_ptr, int32_t **col_idx,
                              double **val) {
  return mmio_read_impl(path, m, n, nnz, is_symmetric, row_ptr, col_idx, val, true);
}

pf_status pf_mmio_read_cached(const char *mtx_path, const char *cache_path, int64_t *m,
                              int64_t *n, int64_t *nnz, int *is_symmetric, int64_t **row_ptr,
                              int32_t **col_idx, double **val, int *from_cache) {
  return mmio_read_cached_impl(mtx_path, cache_path, m, n, nnz, is_symmetric, row_ptr, col_idx,
                               val, from_cache, false);
}

pf_status pf_mmio_read_cached_pinned(const char *mtx_path, const char *cache_path, int64_t *m,
                                     int64_t *n, int64_t *nnz, int *is_symmetric,
                                     int64_t **row_ptr, int32_t **col_idx, double **val,
                                     int *from_cache) {
  return mmio_read_cached_impl(mtx_path, cache_path, m, n, nnz, is_symmetric, row_ptr, col_idx,
                               val, from_cache, true);
}

pf_status pf_shard_bounds_i32(const int32_t *row_ptr, int64_t m, int parts, int64_t *bounds) {
  return shard_bounds(row_ptr, m, parts, bounds);
}
pf_status pf_shard_bounds_i64(const int64_t *row_ptr, int64_t m, int parts, int64_t *bounds) {
  return shard_bounds(row_ptr, m, parts, bounds);
}

}  // extern "C"
