// Host half of libsc_b200.so: Matrix-Market and .cfmtx I/O, the pattern
// dictionary, and the enumerate + coarsen conversion (CSR -> CF).
//
// The conversion follows code_gen/ss_format/format_generator.py:36-129 of the
// reference step for step (same merge order, same padding rules) but runs as
// native code, one row panel per task, with panels spread over host threads.

#include <algorithm>
#include <charconv>
#include <cerrno>
#include <cinttypes>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <memory>
#include <sstream>
#include <thread>
#include <unordered_map>

#include "sc_internal.h"

// ------------------------------------------------------------------ errors --

static thread_local std::string g_last_error;

void sc_set_error(const std::string &msg) { g_last_error = msg; }
void sc_clear_error() { g_last_error.clear(); }

extern "C" const char *sc_last_error_string(void) { return g_last_error.c_str(); }
extern "C" int sc_version(void) { return 100; }  // 0.1.0

#define SC_API_BEGIN try {
#define SC_API_END                                  \
  }                                                 \
  catch (const sc_error &e) {                       \
    sc_set_error(e.what());                         \
    return e.code;                                  \
  }                                                 \
  catch (const std::bad_alloc &) {                  \
    sc_set_error("host allocation failed");         \
    return SC_ERR_NOMEM;                            \
  }                                                 \
  catch (const std::exception &e) {                 \
    sc_set_error(e.what());                         \
    return SC_ERR_ARG;                              \
  }                                                 \
  return SC_OK;

static void require(bool cond, int code, const std::string &msg) {
  if (!cond) throw sc_error(code, msg);
}

// ----------------------------------------------------------- float repr --

// Python's float repr: the shortest decimal string that round-trips to the
// same double, laid out in fixed notation when the decimal exponent is in
// [-4, 16) and in scientific notation ("1e-05", "1.5e+16") otherwise.  numpy
// float64 str() uses the same rule; format_writer relies on it
// (format_generator.py:157).
std::string sc_py_float_repr(double d) {
  if (std::isnan(d)) return "nan";
  if (std::isinf(d)) return d < 0 ? "-inf" : "inf";
  if (d == 0.0) return std::signbit(d) ? "-0.0" : "0.0";
  // Shortest round-trip digits in scientific form (std::to_chars, i.e. the
  // Ryu algorithm in libstdc++), then Python's layout below.
  char buf[64];
  auto res = std::to_chars(buf, buf + sizeof buf - 1, d, std::chars_format::scientific);
  *res.ptr = '\0';
  // buf = [-]D[.DDD]e[+-]XX
  std::string s(buf);
  bool neg = s[0] == '-';
  if (neg) s = s.substr(1);
  size_t epos = s.find('e');
  int exp10 = atoi(s.c_str() + epos + 1);
  std::string digits;
  for (size_t i = 0; i < epos; ++i)
    if (s[i] != '.') digits.push_back(s[i]);
  while (digits.size() > 1 && digits.back() == '0') digits.pop_back();
  std::string out;
  if (exp10 >= -4 && exp10 < 16) {
    int nd = (int)digits.size();
    if (exp10 < 0) {
      out = "0." + std::string(-exp10 - 1, '0') + digits;
    } else if (exp10 + 1 >= nd) {
      out = digits + std::string(exp10 + 1 - nd, '0') + ".0";
    } else {
      out = digits.substr(0, exp10 + 1) + "." + digits.substr(exp10 + 1);
    }
  } else {
    out = digits.substr(0, 1);
    if (digits.size() > 1) out += "." + digits.substr(1);
    char eb[16];
    snprintf(eb, sizeof eb, "e%c%02d", exp10 < 0 ? '-' : '+', std::abs(exp10));
    out += eb;
  }
  return neg ? "-" + out : out;
}

// ------------------------------------------------------------ file slurp --

static std::string read_file(const char *path) {
  require(path != nullptr, SC_ERR_ARG, "null path");
  FILE *f = fopen(path, "rb");
  require(f != nullptr, SC_ERR_IO, std::string("unable to open file ") + path);
  std::string data;
  char buf[1 << 16];
  size_t n;
  while ((n = fread(buf, 1, sizeof buf, f)) > 0) data.append(buf, n);
  bool err = ferror(f);
  fclose(f);
  require(!err, SC_ERR_IO, std::string("read error on ") + path);
  return data;
}

// Splits text into lines without copying (views into `data`).
struct LineReader {
  const std::string &d;
  size_t pos = 0;
  explicit LineReader(const std::string &s) : d(s) {}
  bool next(const char *&b, const char *&e) {
    if (pos >= d.size()) return false;
    size_t nl = d.find('\n', pos);
    if (nl == std::string::npos) nl = d.size();
    b = d.data() + pos;
    e = d.data() + nl;
    if (e > b && e[-1] == '\r') --e;
    pos = nl + 1;
    return true;
  }
};

static inline const char *skip_ws(const char *p, const char *e) {
  while (p < e && (*p == ' ' || *p == '\t')) ++p;
  return p;
}

// --------------------------------------------------------------- .mtx ----

// Reads a coordinate Matrix-Market file.  Header handling follows sym_lib's
// read_header (aggregation/utils/sparse_io.cpp:278-339): real | integer |
// pattern, general | symmetric; complex, array and skew/hermitian are
// rejected.  Entries are 1-based; symmetric files are expanded (off-diagonal
// mirrored) as sym_lib's make_full and scipy's mmread both do.  The CSR has
// columns ascending in every row; duplicate coordinates are summed and
// explicit zeros are kept, which is what scipy's mmread(...).tocsr() gives
// the reference converter (format_generator.py:214-215).
static sc_csr *load_mtx(const char *path) {
  std::string data = read_file(path);
  LineReader lr(data);
  const char *b, *e;
  require(lr.next(b, e), SC_ERR_FORMAT, "empty .mtx file");
  std::string banner(b, e);
  for (auto &c : banner) c = (char)tolower((unsigned char)c);
  std::istringstream iss(banner);
  std::string t0, t1, t2, t3, t4;
  require((bool)(iss >> t0 >> t1 >> t2 >> t3 >> t4), SC_ERR_FORMAT,
          "first line does not contain 5 tokens");
  require(t0 == "%%matrixmarket", SC_ERR_FORMAT, "first token is not %%MatrixMarket");
  require(t1 == "matrix", SC_ERR_FORMAT, "not a matrix");
  require(t2 == "coordinate", SC_ERR_FORMAT, "only coordinate .mtx files are supported");
  bool pattern = false;
  if (t3 == "pattern") pattern = true;
  else require(t3 == "real" || t3 == "integer", SC_ERR_FORMAT, "unsupported arithmetic: " + t3);
  bool symmetric = false;
  if (t4 == "symmetric") symmetric = true;
  else require(t4 == "general", SC_ERR_FORMAT, "unsupported shape: " + t4);

  long long m = -1, n = -1, nnz = -1;
  while (lr.next(b, e)) {
    const char *p = skip_ws(b, e);
    if (p == e || *p == '%') continue;
    std::string l(p, e);
    require(sscanf(l.c_str(), "%lld %lld %lld", &m, &n, &nnz) == 3, SC_ERR_FORMAT,
            "the matrix dimension is missing");
    break;
  }
  require(m >= 0 && n >= 0 && nnz >= 0, SC_ERR_FORMAT, "the matrix dimension is missing");
  require(m < INT32_MAX && n < INT32_MAX, SC_ERR_UNSUPPORTED, "matrix dimension exceeds int32");

  struct Trip { int32_t r, c; double v; };
  std::vector<Trip> trips;
  trips.reserve((size_t)nnz * (symmetric ? 2 : 1));
  long long got = 0;
  while (got < nnz && lr.next(b, e)) {
    const char *p = skip_ws(b, e);
    if (p == e || *p == '%') continue;
    char *q;
    long long r = strtoll(p, &q, 10);
    require(q != p, SC_ERR_FORMAT, "bad entry line in .mtx");
    p = q;
    long long c = strtoll(p, &q, 10);
    require(q != p, SC_ERR_FORMAT, "bad entry line in .mtx");
    p = q;
    double v = 1.0;
    if (!pattern) {
      v = strtod(p, &q);
      require(q != p, SC_ERR_FORMAT, "missing value in .mtx entry");
    }
    require(r >= 1 && r <= m && c >= 1 && c <= n, SC_ERR_FORMAT, "entry index out of range in .mtx");
    trips.push_back({(int32_t)(r - 1), (int32_t)(c - 1), v});
    if (symmetric && r != c) trips.push_back({(int32_t)(c - 1), (int32_t)(r - 1), v});
    ++got;
  }
  require(got == nnz, SC_ERR_FORMAT, "fewer entries than the header declares");

  auto *a = new sc_csr();
  std::unique_ptr<sc_csr> guard(a);
  a->m = (int32_t)m;
  a->n = (int32_t)n;
  // Counting sort by row, then by column inside each row (stable), then sum
  // duplicates.
  std::vector<int64_t> cnt((size_t)m + 1, 0);
  for (auto &t : trips) cnt[t.r + 1]++;
  for (long long i = 0; i < m; ++i) cnt[i + 1] += cnt[i];
  std::vector<int32_t> cols(trips.size());
  std::vector<double> vals(trips.size());
  {
    std::vector<int64_t> pos(cnt.begin(), cnt.end() - 1);
    for (auto &t : trips) {
      int64_t k = pos[t.r]++;
      cols[k] = t.c;
      vals[k] = t.v;
    }
  }
  trips.clear();
  trips.shrink_to_fit();
  a->rowptr.assign((size_t)m + 1, 0);
  a->colind.reserve(cols.size());
  a->vals.reserve(vals.size());
  std::vector<std::pair<int32_t, double>> row;
  for (long long i = 0; i < m; ++i) {
    row.clear();
    for (int64_t k = cnt[i]; k < cnt[i + 1]; ++k) row.push_back({cols[k], vals[k]});
    std::stable_sort(row.begin(), row.end(),
                     [](const std::pair<int32_t, double> &x, const std::pair<int32_t, double> &y) {
                       return x.first < y.first;
                     });
    for (size_t k = 0; k < row.size(); ++k) {
      if (!a->colind.empty() && (int64_t)a->colind.size() > a->rowptr[i] &&
          a->colind.back() == row[k].first) {
        a->vals.back() += row[k].second;
      } else {
        a->colind.push_back(row[k].first);
        a->vals.push_back(row[k].second);
      }
    }
    require(a->colind.size() < (size_t)INT32_MAX, SC_ERR_UNSUPPORTED, "nnz exceeds int32");
    a->rowptr[i + 1] = (int32_t)a->colind.size();
  }
  return guard.release();
}

// -------------------------------------------------------------- .cfmtx ---

static bool is_pad_token(const std::string &t) {
  // format_writer prints coarsening padding as the Python int 0 -> "0"; real
  // values are float64 reprs, which always carry '.', 'e', "nan" or "inf".
  return t.find_first_not_of("+-0123456789") == std::string::npos;
}

static void parse_int_line(const char *b, const char *e, std::vector<int32_t> &out) {
  const char *p = b;
  while (true) {
    p = skip_ws(p, e);
    if (p >= e) break;
    char *q;
    long long v = strtoll(p, &q, 10);
    require(q != p && (q == e || *q == ' ' || *q == '\t'), SC_ERR_FORMAT,
            "non-integer token in .cfmtx integer line");
    require(v >= INT32_MIN && v <= INT32_MAX, SC_ERR_FORMAT, "integer out of int32 range in .cfmtx");
    out.push_back((int32_t)v);
    p = q;
  }
}

// Parses a .cfmtx (layout of format_writer, format_generator.py:132-160;
// reader semantics of readCFMTXFile, utils/Sparse_io.cpp:84-181).
static sc_cf *load_cfmtx(const char *path) {
  std::string data = read_file(path);
  LineReader lr(data);
  const char *b, *e;
  auto *cf = new sc_cf();
  std::unique_ptr<sc_cf> guard(cf);
  cf->from_text = true;
  require(lr.next(b, e), SC_ERR_FORMAT, "empty .cfmtx file");
  {
    std::string l(b, e);
    int np = 0;
    require(sscanf(l.c_str(), "%d %d %d %d %d", &cf->num_rows, &cf->num_cols, &cf->kernel_m, &np,
                   &cf->vector_length_hdr) == 5,
            SC_ERR_FORMAT, ".cfmtx header must hold 5 integers");
    require(np >= 0 && cf->num_rows >= 0 && cf->num_cols >= 0 && cf->kernel_m >= 1, SC_ERR_FORMAT,
            "bad .cfmtx header");
    cf->header.resize(np);
    cf->pats.resize(np);
  }
  const int np = (int)cf->pats.size();
  for (int i = 0; i < np; ++i) {
    require(lr.next(b, e), SC_ERR_FORMAT, "truncated .cfmtx pattern list");
    std::string l(b, e);
    char mask[256];
    int id = -1;
    require(sscanf(l.c_str(), "%255s %d", mask, &id) == 2, SC_ERR_FORMAT, "bad pattern line in .cfmtx");
    cf->header[i] = {mask, id};
  }
  // Body block i belongs to pattern id i.  When the header's ids are a
  // permutation of 0..np-1 the block takes the mask of that id; otherwise the
  // header position is used, as readCFMTXFile does (Sparse_io.cpp:101-133).
  std::vector<int> by_id(np, -1);
  bool perm = true;
  for (int i = 0; i < np; ++i) {
    int id = cf->header[i].second;
    if (id < 0 || id >= np || by_id[id] != -1) { perm = false; break; }
    by_id[id] = i;
  }
  for (int i = 0; i < np; ++i) {
    sc_pattern &pt = cf->pats[i];
    pt.mask = cf->header[perm ? by_id[i] : i].first;
    pt.popcount = (int32_t)std::count(pt.mask.begin(), pt.mask.end(), '1');
    require(lr.next(b, e), SC_ERR_FORMAT, "truncated .cfmtx body (RPP line)");
    parse_int_line(b, e, pt.rpp);
    require(lr.next(b, e), SC_ERR_FORMAT, "truncated .cfmtx body (CB line)");
    parse_int_line(b, e, pt.cb);
    require(lr.next(b, e), SC_ERR_FORMAT, "truncated .cfmtx body (values line)");
    const char *p = b;
    while (true) {
      p = skip_ws(p, e);
      if (p >= e) break;
      const char *q = p;
      while (q < e && *q != ' ' && *q != '\t') ++q;
      std::string tok(p, q);
      char *endp;
      // readCFMTXFile reads values with `istream >> float`, i.e. the decimal
      // text is rounded straight to float32.
      float fv = strtof(tok.c_str(), &endp);
      require(endp != tok.c_str() && *endp == '\0', SC_ERR_FORMAT, "bad value token in .cfmtx: " + tok);
      pt.vals.push_back(fv);
      pt.vals_d.push_back(strtod(tok.c_str(), nullptr));
      bool pad = is_pad_token(tok);
      pt.pad.push_back(pad ? 1 : 0);
      if (!pad) cf->real_nnz++;
      pt.tokens.push_back(std::move(tok));
      p = q;
    }
  }
  return guard.release();
}

static void write_cfmtx(const sc_cf *cf, const char *path) {
  require(path != nullptr, SC_ERR_ARG, "null path");
  FILE *f = fopen(path, "wb");
  require(f != nullptr, SC_ERR_IO, std::string("unable to open file for writing ") + path);
  std::string buf;
  buf.reserve(1 << 20);
  auto flush = [&]() {
    if (!buf.empty()) {
      size_t w = fwrite(buf.data(), 1, buf.size(), f);
      if (w != buf.size()) {
        fclose(f);
        throw sc_error(SC_ERR_IO, std::string("write error on ") + path);
      }
      buf.clear();
    }
  };
  char tmp[64];
  snprintf(tmp, sizeof tmp, "%d %d %d %d %d\n", cf->num_rows, cf->num_cols, cf->kernel_m,
           (int)cf->header.size(), cf->vector_length_hdr);
  buf += tmp;
  for (auto &h : cf->header) {
    buf += h.first;
    snprintf(tmp, sizeof tmp, " %d \n", h.second);
    buf += tmp;
  }
  auto put_ints = [&](const std::vector<int32_t> &v) {
    for (size_t i = 0; i < v.size(); ++i) {
      if (i) buf.push_back(' ');
      snprintf(tmp, sizeof tmp, "%d", v[i]);
      buf += tmp;
      if (buf.size() > (1u << 20)) flush();
    }
    buf.push_back('\n');
  };
  for (auto &pt : cf->pats) {
    put_ints(pt.rpp);
    put_ints(pt.cb);
    for (size_t i = 0; i < pt.vals.size(); ++i) {
      if (i) buf.push_back(' ');
      if (cf->from_text) buf += pt.tokens[i];
      else if (pt.pad[i]) buf.push_back('0');
      else buf += sc_py_float_repr(pt.vals_d[i]);
      if (buf.size() > (1u << 20)) flush();
    }
    buf.push_back('\n');
  }
  flush();
  bool err = fclose(f) != 0;
  require(!err, SC_ERR_IO, std::string("close error on ") + path);
}

// ------------------------------------------------------ binary sidecar ----

// Binary companion of a .cfmtx ("<file>.cfbin"): the same content as raw
// little-endian arrays, every array starting on a 16-byte boundary, so
// loading is a few large reads instead of parsing ~10 text tokens per
// nonzero.  Layout:
//   "SCCFBIN1" | i32 num_rows, num_cols, kernel_m, num_patterns, vector_length,
//   i32 0 | i64 real_nnz | per header line: i32 id, i32 len, mask bytes |
//   per pattern (pad to 16): i32 popcount, i32 mask_len, i64 n_rpp, n_cb, n_vals,
//   mask bytes, then (each padded to 16) rpp i32[], cb i32[], vals f32[],
//   vals_d f64[], pad u8[].
static const char kBinMagic[8] = {'S', 'C', 'C', 'F', 'B', 'I', 'N', '1'};

static void write_cfbin(const sc_cf *cf, const char *path) {
  require(path != nullptr, SC_ERR_ARG, "null path");
  FILE *f = fopen(path, "wb");
  require(f != nullptr, SC_ERR_IO, std::string("unable to open file for writing ") + path);
  size_t pos = 0;
  bool ok = true;
  auto put = [&](const void *p, size_t n) {
    if (n && fwrite(p, 1, n, f) != n) ok = false;
    pos += n;
  };
  auto align16 = [&]() {
    static const char z[16] = {0};
    if (pos % 16) put(z, 16 - pos % 16);
  };
  put(kBinMagic, 8);
  int32_t h[6] = {cf->num_rows, cf->num_cols, cf->kernel_m, (int32_t)cf->header.size(), cf->vector_length_hdr, 0};
  put(h, sizeof h);
  put(&cf->real_nnz, 8);
  for (auto &l : cf->header) {
    int32_t x[2] = {l.second, (int32_t)l.first.size()};
    put(x, 8);
    put(l.first.data(), l.first.size());
  }
  for (auto &pt : cf->pats) {
    align16();
    int32_t a[2] = {pt.popcount, (int32_t)pt.mask.size()};
    int64_t b[3] = {(int64_t)pt.rpp.size(), (int64_t)pt.cb.size(), (int64_t)pt.vals.size()};
    put(a, 8);
    put(b, 24);
    put(pt.mask.data(), pt.mask.size());
    align16(); put(pt.rpp.data(), pt.rpp.size() * 4);
    align16(); put(pt.cb.data(), pt.cb.size() * 4);
    align16(); put(pt.vals.data(), pt.vals.size() * 4);
    align16(); put(pt.vals_d.data(), pt.vals_d.size() * 8);
    align16(); put(pt.pad.data(), pt.pad.size());
  }
  ok = (fclose(f) == 0) && ok;
  require(ok, SC_ERR_IO, std::string("write error on ") + path);
}

static sc_cf *load_cfbin(const char *path) {
  std::string d = read_file(path);
  size_t pos = 0;
  auto get = [&](void *p, size_t n) {
    require(pos + n <= d.size(), SC_ERR_FORMAT, "truncated .cfbin file");
    if (n) memcpy(p, d.data() + pos, n);
    pos += n;
  };
  auto align16 = [&]() { pos = (pos + 15) & ~(size_t)15; };
  char magic[8];
  get(magic, 8);
  require(memcmp(magic, kBinMagic, 8) == 0, SC_ERR_FORMAT, "not a .cfbin file (bad magic)");
  auto *cf = new sc_cf();
  std::unique_ptr<sc_cf> guard(cf);
  int32_t h[6];
  get(h, sizeof h);
  cf->num_rows = h[0]; cf->num_cols = h[1]; cf->kernel_m = h[2]; cf->vector_length_hdr = h[4];
  require(h[3] >= 0 && h[0] >= 0 && h[1] >= 0 && h[2] >= 1, SC_ERR_FORMAT, "bad .cfbin header");
  get(&cf->real_nnz, 8);
  cf->header.resize(h[3]);
  cf->pats.resize(h[3]);
  for (auto &l : cf->header) {
    int32_t x[2];
    get(x, 8);
    require(x[1] >= 0 && x[1] < 4096, SC_ERR_FORMAT, "bad mask length in .cfbin");
    l.second = x[0];
    l.first.assign((size_t)x[1], '0');
    get(&l.first[0], (size_t)x[1]);
  }
  for (auto &pt : cf->pats) {
    align16();
    int32_t a[2];
    int64_t b[3];
    get(a, 8);
    get(b, 24);
    require(a[1] >= 0 && a[1] < 4096 && b[0] >= 0 && b[1] >= 0 && b[2] >= 0 &&
                (size_t)(b[0] + b[1] + b[2]) <= d.size(),
            SC_ERR_FORMAT, "bad pattern sizes in .cfbin");
    pt.popcount = a[0];
    pt.mask.assign((size_t)a[1], '0');
    get(&pt.mask[0], (size_t)a[1]);
    pt.rpp.resize(b[0]); pt.cb.resize(b[1]); pt.vals.resize(b[2]); pt.vals_d.resize(b[2]); pt.pad.resize(b[2]);
    align16(); get(pt.rpp.data(), b[0] * 4);
    align16(); get(pt.cb.data(), b[1] * 4);
    align16(); get(pt.vals.data(), b[2] * 4);
    align16(); get(pt.vals_d.data(), b[2] * 8);
    align16(); get(pt.pad.data(), b[2]);
  }
  return guard.release();
}

// ----------------------------------------------------- pattern dictionary --

// Dictionary in Python-dict semantics: `order` is the insertion order of the
// patterns dict built in format_generator.py:200-208, and lookup maps a row
// mask (bit j = panel row j) to its id.
struct PatternDict {
  int m = 0;
  std::vector<std::pair<std::string, int32_t>> order;
  std::vector<int32_t> table;                    // dense lookup for m <= 20
  std::unordered_map<uint64_t, int32_t> sparse;  // m > 20
  int32_t lookup(uint64_t rowmask) const {
    if (!table.empty()) return table[rowmask];
    auto it = sparse.find(rowmask);
    return it == sparse.end() ? -1 : it->second;
  }
};

static uint64_t mask_string_to_rowbits(const std::string &s) {
  uint64_t bits = 0;
  for (size_t j = 0; j < s.size(); ++j)
    if (s[j] == '1') bits |= (uint64_t)1 << j;
  return bits;
}

// build_patterns_map(m, 1) (pattern_dictionary.py:29-37): id i-1 <-> the
// m-bit binary string of 2^m - i, panel row 0 being the leftmost character.
static PatternDict default_dict(int m) {
  PatternDict d;
  d.m = m;
  uint64_t full = ((uint64_t)1 << m);
  for (uint64_t i = 1; i < full; ++i) {
    uint64_t x = full - i;
    std::string s(m, '0');
    for (int j = 0; j < m; ++j)
      if (x >> (m - 1 - j) & 1) s[j] = '1';
    d.order.push_back({s, (int32_t)(i - 1)});
  }
  return d;
}

// read_pattern_dictionary (pattern_dictionary.py:49-60) followed by the
// patterns dict construction of format_generator.py:200-206: lines "<mask>
// <id>" after a 3-token first line; a repeated id keeps its first position and
// takes the last mask; a repeated mask maps to its last id.
static PatternDict read_dict_file(const char *path, int m) {
  std::string data = read_file(path);
  LineReader lr(data);
  const char *b, *e;
  require(lr.next(b, e), SC_ERR_FORMAT, "empty pattern dictionary");
  {
    std::istringstream iss(std::string(b, e));
    std::string a1, a2, a3;
    require((bool)(iss >> a1 >> a2 >> a3), SC_ERR_FORMAT, "dictionary first line needs 3 tokens");
  }
  std::vector<int32_t> id_order;
  std::unordered_map<int32_t, std::string> id_to_mask;
  while (lr.next(b, e)) {
    std::istringstream iss(std::string(b, e));
    std::string mask, extra;
    long long id;
    if (!(iss >> mask)) continue;  // blank line
    require((bool)(iss >> id) && !(iss >> extra), SC_ERR_FORMAT, "dictionary line must be '<mask> <id>'");
    if (!id_to_mask.count((int32_t)id)) id_order.push_back((int32_t)id);
    id_to_mask[(int32_t)id] = mask;
  }
  PatternDict d;
  d.m = m;
  std::vector<std::string> seen_masks;
  std::unordered_map<std::string, size_t> mask_pos;
  std::vector<std::pair<std::string, int32_t>> order;
  for (int32_t id : id_order) {
    // Python: patterns[tuple(mask == '1')] = id; keys are boolean tuples, so
    // masks are compared after mapping non-'1' characters to '0'.
    std::string norm = id_to_mask[id];
    for (auto &c : norm) c = (c == '1') ? '1' : '0';
    auto it = mask_pos.find(norm);
    if (it == mask_pos.end()) {
      mask_pos[norm] = order.size();
      order.push_back({id_to_mask[id], id});
    } else {
      order[it->second].second = id;
    }
  }
  d.order = order;
  return d;
}

static void finish_dict(PatternDict &d) {
  const int m = d.m;
  const int np = (int)d.order.size();
  for (auto &o : d.order) {
    require(o.second >= 0 && o.second < np, SC_ERR_FORMAT,
            "pattern ids must lie in [0, number of patterns)");
    require(std::count(o.first.begin(), o.first.end(), '1') > 0, SC_ERR_FORMAT,
            "a pattern with no nonzero row cannot be packed");
  }
  if (m <= 20) d.table.assign((size_t)1 << m, -1);
  for (auto &o : d.order) {
    if ((int)o.first.size() != m) continue;  // tuple length differs: never matches
    uint64_t bits = mask_string_to_rowbits(o.first);
    if (m <= 20) d.table[bits] = o.second;
    else d.sparse[bits] = o.second;
  }
}

// ----------------------------------------------------- enumerate+coarsen --

struct ChunkOut {
  // per pattern id: padded column list, values, pad flags, and per-panel
  // padded column counts
  std::vector<std::vector<int32_t>> cb;
  std::vector<std::vector<double>> vals;
  std::vector<std::vector<uint8_t>> pad;
  std::vector<std::vector<int32_t>> panel_len;
  int64_t real = 0;
};

// One row panel, as the body of the `for start_row` loop in
// format_generator.py:93-127: a k-way merge over the panel's rows by column;
// at each step the rows whose current column equals the minimum form the
// pattern; the column and the matched rows' values (row order) go to that
// pattern's list; then transform_row_panel (format_generator.py:36-65) pads
// values with 0 to a multiple of pack*popcount and columns with the list's
// maximum to a multiple of pack.
static void coarsen_panels(const sc_csr &a, const PatternDict &d, const std::vector<int> &popc,
                           int m, int kernel_n, int64_t p0, int64_t p1, ChunkOut &out) {
  const int np = (int)d.order.size();
  out.cb.assign(np, {});
  out.vals.assign(np, {});
  out.pad.assign(np, {});
  out.panel_len.assign(np, {});
  std::vector<std::vector<int32_t>> pcols(np);
  std::vector<std::vector<double>> pvals(np);
  std::vector<int64_t> ptr(m), end(m);
  for (int64_t p = p0; p < p1; ++p) {
    for (int id = 0; id < np; ++id) { pcols[id].clear(); pvals[id].clear(); }
    for (int r = 0; r < m; ++r) {
      int64_t row = p * m + r;
      if (row < a.m) { ptr[r] = a.rowptr[row]; end[r] = a.rowptr[row + 1]; }
      else { ptr[r] = end[r] = 0; }
    }
    while (true) {
      int32_t mn = INT32_MAX;
      bool any = false;
      for (int r = 0; r < m; ++r)
        if (ptr[r] < end[r]) { any = true; mn = std::min(mn, a.colind[ptr[r]]); }
      if (!any) break;
      uint64_t bits = 0;
      for (int r = 0; r < m; ++r)
        if (ptr[r] < end[r] && a.colind[ptr[r]] == mn) bits |= (uint64_t)1 << r;
      int32_t id = d.lookup(bits);
      if (id >= 0) {
        pcols[id].push_back(mn);
        for (int r = 0; r < m; ++r)
          if (bits >> r & 1) pvals[id].push_back(a.vals[ptr[r]]);
      }
      for (int r = 0; r < m; ++r)
        if (bits >> r & 1) ptr[r]++;
    }
    for (int id = 0; id < np; ++id) {
      const int P = popc[id];
      const int pack = kernel_n == 0 ? 32 / P : kernel_n;
      auto &c = pcols[id];
      auto &v = pvals[id];
      out.real += (int64_t)v.size();
      out.vals[id].insert(out.vals[id].end(), v.begin(), v.end());
      out.pad[id].insert(out.pad[id].end(), v.size(), 0);
      size_t rem = v.size() % (size_t)(pack * P);
      if (!v.empty() && rem != 0) {
        size_t add = (size_t)(pack * P) - rem;
        out.vals[id].insert(out.vals[id].end(), add, 0.0);
        out.pad[id].insert(out.pad[id].end(), add, 1);
      }
      out.cb[id].insert(out.cb[id].end(), c.begin(), c.end());
      size_t remc = c.size() % (size_t)pack;
      size_t len = c.size();
      if (!c.empty() && remc != 0) {
        int32_t cmax = *std::max_element(c.begin(), c.end());
        out.cb[id].insert(out.cb[id].end(), pack - remc, cmax);
        len += pack - remc;
      }
      out.panel_len[id].push_back((int32_t)len);
    }
  }
}

static sc_cf *coarsen(const sc_csr &a, int m, int kernel_n, const char *dict_path, int nthreads) {
  require(m >= 1 && m <= 30, SC_ERR_UNSUPPORTED, "kernel_m must be in 1..30");
  require(kernel_n >= 0, SC_ERR_ARG, "kernel_n must be >= 0");
  PatternDict d = (dict_path == nullptr || strcmp(dict_path, "false") == 0)
                      ? default_dict(m)
                      : read_dict_file(dict_path, m);
  finish_dict(d);
  const int np = (int)d.order.size();
  // Body block i is the pattern whose id is i.
  std::vector<int> popc(np, 0);
  std::vector<std::string> mask_of(np);
  for (auto &o : d.order) {
    mask_of[o.second] = o.first;
    popc[o.second] = (int)std::count(o.first.begin(), o.first.end(), '1');
  }
  for (int id = 0; id < np; ++id) {
    require(!mask_of[id].empty(), SC_ERR_FORMAT, "pattern ids must be 0..number_of_patterns-1");
    require(kernel_n != 0 || popc[id] <= 32, SC_ERR_UNSUPPORTED,
            "kernel_n == 0 needs every pattern popcount <= 32");
  }
  const int64_t panels = ((int64_t)a.m + m - 1) / m;
  int T = nthreads > 0 ? nthreads : (int)std::max(1u, std::thread::hardware_concurrency());
  T = (int)std::max<int64_t>(1, std::min<int64_t>(T, panels / 16 + 1));
  std::vector<ChunkOut> chunks(T);
  {
    std::vector<std::thread> th;
    std::vector<std::string> errs(T);
    for (int t = 0; t < T; ++t) {
      int64_t p0 = panels * t / T, p1 = panels * (t + 1) / T;
      th.emplace_back([&, t, p0, p1]() {
        try { coarsen_panels(a, d, popc, m, kernel_n, p0, p1, chunks[t]); }
        catch (const std::exception &ex) { errs[t] = ex.what(); }
      });
    }
    for (auto &x : th) x.join();
    for (auto &s : errs) require(s.empty(), SC_ERR_NOMEM, s);
  }
  auto *cf = new sc_cf();
  std::unique_ptr<sc_cf> guard(cf);
  cf->num_rows = a.m;
  cf->num_cols = a.n;
  cf->kernel_m = m;
  cf->vector_length_hdr = kernel_n;
  cf->header = d.order;
  cf->pats.resize(np);
  for (int id = 0; id < np; ++id) {
    sc_pattern &pt = cf->pats[id];
    pt.mask = mask_of[id];
    pt.popcount = popc[id];
    size_t ncb = 0, nv = 0;
    for (auto &c : chunks) { ncb += c.cb[id].size(); nv += c.vals[id].size(); }
    require(ncb < (size_t)INT32_MAX, SC_ERR_UNSUPPORTED, "pattern block exceeds int32 indexing");
    pt.cb.reserve(ncb);
    pt.vals_d.reserve(nv);
    pt.pad.reserve(nv);
    pt.rpp.reserve(panels + 1);
    pt.rpp.push_back(0);
    for (auto &c : chunks) {
      pt.cb.insert(pt.cb.end(), c.cb[id].begin(), c.cb[id].end());
      pt.vals_d.insert(pt.vals_d.end(), c.vals[id].begin(), c.vals[id].end());
      pt.pad.insert(pt.pad.end(), c.pad[id].begin(), c.pad[id].end());
      for (int32_t len : c.panel_len[id]) pt.rpp.push_back(pt.rpp.back() + len);
      std::vector<int32_t>().swap(c.cb[id]);
      std::vector<double>().swap(c.vals[id]);
      std::vector<uint8_t>().swap(c.pad[id]);
    }
    pt.vals.resize(pt.vals_d.size());
    for (size_t i = 0; i < pt.vals_d.size(); ++i) pt.vals[i] = (float)pt.vals_d[i];
  }
  for (auto &c : chunks) cf->real_nnz += c.real;
  return guard.release();
}

// -------------------------------------------------------------- C ABI ----

extern "C" {

int sc_mtx_load_csr(const char *mtx_path, sc_csr **out) {
  SC_API_BEGIN
  require(out != nullptr, SC_ERR_ARG, "null output handle");
  *out = load_mtx(mtx_path);
  SC_API_END
}

int sc_csr_create(int32_t m, int32_t n, int64_t nnz, const int32_t *rowptr, const int32_t *colind,
                  const double *vals, sc_csr **out) {
  SC_API_BEGIN
  require(out != nullptr && rowptr != nullptr, SC_ERR_ARG, "null argument");
  require(m >= 0 && n >= 0 && nnz >= 0 && nnz < INT32_MAX, SC_ERR_ARG, "bad CSR sizes");
  require(nnz == 0 || (colind != nullptr && vals != nullptr), SC_ERR_ARG, "null CSR arrays");
  require(rowptr[0] == 0 && rowptr[m] == nnz, SC_ERR_ARG, "rowptr must start at 0 and end at nnz");
  for (int32_t i = 0; i < m; ++i) {
    require(rowptr[i] <= rowptr[i + 1], SC_ERR_ARG, "rowptr must be non-decreasing");
    for (int32_t k = rowptr[i]; k < rowptr[i + 1]; ++k) {
      require(colind[k] >= 0 && colind[k] < n, SC_ERR_ARG, "column index out of range");
      require(k == rowptr[i] || colind[k] > colind[k - 1], SC_ERR_ARG,
              "columns must be strictly ascending inside each row");
    }
  }
  auto a = std::make_unique<sc_csr>();
  a->m = m;
  a->n = n;
  a->rowptr.assign(rowptr, rowptr + m + 1);
  a->colind.assign(colind, colind + nnz);
  a->vals.assign(vals, vals + nnz);
  *out = a.release();
  SC_API_END
}

int sc_csr_dims(const sc_csr *a, int32_t *m, int32_t *n, int64_t *nnz) {
  SC_API_BEGIN
  require(a != nullptr, SC_ERR_ARG, "null CSR handle");
  if (m) *m = a->m;
  if (n) *n = a->n;
  if (nnz) *nnz = (int64_t)a->colind.size();
  SC_API_END
}

int sc_csr_arrays(const sc_csr *a, const int32_t **rowptr, const int32_t **colind, const double **vals) {
  SC_API_BEGIN
  require(a != nullptr, SC_ERR_ARG, "null CSR handle");
  if (rowptr) *rowptr = a->rowptr.data();
  if (colind) *colind = a->colind.data();
  if (vals) *vals = a->vals.data();
  SC_API_END
}

void sc_csr_free(sc_csr *a) { delete a; }

int sc_cf_load(const char *cfmtx_path, sc_cf **out) {
  SC_API_BEGIN
  require(out != nullptr, SC_ERR_ARG, "null output handle");
  *out = load_cfmtx(cfmtx_path);
  SC_API_END
}

int sc_cf_from_csr(const sc_csr *a, int32_t kernel_m, int32_t kernel_n, const char *dict_path,
                   int32_t nthreads, sc_cf **out) {
  SC_API_BEGIN
  require(a != nullptr && out != nullptr, SC_ERR_ARG, "null argument");
  *out = coarsen(*a, kernel_m, kernel_n, dict_path, nthreads);
  SC_API_END
}

int sc_cf_write(const sc_cf *cf, const char *path) {
  SC_API_BEGIN
  require(cf != nullptr, SC_ERR_ARG, "null CF handle");
  write_cfmtx(cf, path);
  SC_API_END
}

int sc_cf_write_binary(const sc_cf *cf, const char *path) {
  SC_API_BEGIN
  require(cf != nullptr, SC_ERR_ARG, "null CF handle");
  write_cfbin(cf, path);
  SC_API_END
}

int sc_cf_load_binary(const char *path, sc_cf **out) {
  SC_API_BEGIN
  require(out != nullptr, SC_ERR_ARG, "null output handle");
  *out = load_cfbin(path);
  SC_API_END
}

int sc_cf_dims(const sc_cf *cf, int32_t *num_rows, int32_t *num_cols, int32_t *kernel_m,
               int32_t *num_patterns, int32_t *vector_length) {
  SC_API_BEGIN
  require(cf != nullptr, SC_ERR_ARG, "null CF handle");
  if (num_rows) *num_rows = cf->num_rows;
  if (num_cols) *num_cols = cf->num_cols;
  if (kernel_m) *kernel_m = cf->kernel_m;
  if (num_patterns) *num_patterns = (int32_t)cf->pats.size();
  if (vector_length) *vector_length = cf->vector_length_hdr;
  SC_API_END
}

int sc_cf_header_line(const sc_cf *cf, int32_t line, char *mask_out, int32_t mask_cap, int32_t *pattern_id) {
  SC_API_BEGIN
  require(cf != nullptr, SC_ERR_ARG, "null CF handle");
  require(line >= 0 && line < (int32_t)cf->header.size(), SC_ERR_ARG, "header line out of range");
  const auto &h = cf->header[line];
  if (mask_out) {
    require(mask_cap > (int32_t)h.first.size(), SC_ERR_ARG, "mask buffer too small");
    memcpy(mask_out, h.first.c_str(), h.first.size() + 1);
  }
  if (pattern_id) *pattern_id = h.second;
  SC_API_END
}

int sc_cf_pattern_sizes(const sc_cf *cf, int32_t pattern_id, int32_t *popcount, int64_t *n_rpp,
                        int64_t *n_cb, int64_t *n_vals) {
  SC_API_BEGIN
  require(cf != nullptr, SC_ERR_ARG, "null CF handle");
  require(pattern_id >= 0 && pattern_id < (int32_t)cf->pats.size(), SC_ERR_ARG, "pattern id out of range");
  const auto &p = cf->pats[pattern_id];
  if (popcount) *popcount = p.popcount;
  if (n_rpp) *n_rpp = (int64_t)p.rpp.size();
  if (n_cb) *n_cb = (int64_t)p.cb.size();
  if (n_vals) *n_vals = (int64_t)p.vals.size();
  SC_API_END
}

int sc_cf_pattern_arrays(const sc_cf *cf, int32_t pattern_id, const int32_t **rpp, const int32_t **cb,
                         const float **vals) {
  SC_API_BEGIN
  require(cf != nullptr, SC_ERR_ARG, "null CF handle");
  require(pattern_id >= 0 && pattern_id < (int32_t)cf->pats.size(), SC_ERR_ARG, "pattern id out of range");
  const auto &p = cf->pats[pattern_id];
  if (rpp) *rpp = p.rpp.data();
  if (cb) *cb = p.cb.data();
  if (vals) *vals = p.vals.data();
  SC_API_END
}

int sc_cf_real_nnz(const sc_cf *cf, int64_t *nnz) {
  SC_API_BEGIN
  require(cf != nullptr && nnz != nullptr, SC_ERR_ARG, "null argument");
  *nnz = cf->real_nnz;
  SC_API_END
}

void sc_cf_free(sc_cf *cf) { delete cf; }

// companionMtxPathFromCFMTX (utils/Sparse_io.cpp:28-46).
int sc_companion_mtx_path(const char *cfmtx_path, char *out, int32_t cap) {
  SC_API_BEGIN
  require(cfmtx_path != nullptr && out != nullptr, SC_ERR_ARG, "null argument");
  std::string p(cfmtx_path), r;
  const size_t kSuf = 6;
  if (p.size() <= kSuf) {
    r = p;
  } else {
    std::string stem = p.substr(0, p.size() - kSuf);
    size_t last = stem.rfind('-');
    if (last == std::string::npos || last == 0) {
      r = stem + ".mtx";
    } else {
      size_t second = stem.rfind('-', last - 1);
      if (second == std::string::npos) r = stem + ".mtx";
      else r = stem.substr(0, second) + ".mtx";
    }
  }
  require(cap > (int32_t)r.size(), SC_ERR_ARG, "output buffer too small");
  memcpy(out, r.c_str(), r.size() + 1);
  SC_API_END
}

}  // extern "C"
