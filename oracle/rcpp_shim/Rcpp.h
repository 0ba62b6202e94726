// Minimal stand-in for the Rcpp surface used by the reference's CPU sources.
//
// TEST INFRASTRUCTURE ONLY.  This header lets the reference's own CPU
// implementation (tsne_neighbors.cpp, fast_knn_umap.cpp) compile unmodified,
// from where it lies, into oracle/_ref/ so that it can serve as the parity
// checker and the CPU baseline.  Nothing in the product links against it.
//
// It models just enough of R's object system for those two files:
//   * SEXP is a pointer to a tagged object (integer / real / string / list /
//     S4) with an optional dim attribute (column-major matrices);
//   * Rcpp::Vector / Rcpp::Matrix wrap such objects by reference, like Rcpp;
//   * List::create(Named(..) = value, ...) builds a named list;
//   * stop() throws std::runtime_error, warning() is recorded and ignored.
// Objects are owned by a process-wide pool that the harness clears between
// calls (rshim::collect()), which is sufficient for a batch checker.
#pragma once

#include <cmath>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <iostream>
#include <limits>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <utility>
#include <vector>

enum {
  NILSXP = 0,
  LGLSXP = 10,
  INTSXP = 13,
  REALSXP = 14,
  STRSXP = 16,
  VECSXP = 19,
  EXTPTRSXP = 22,
  S4SXP = 25
};

struct SEXPREC {
  int type = NILSXP;
  std::vector<int> ints;          // INTSXP / LGLSXP payload
  std::vector<double> reals;      // REALSXP payload
  std::vector<std::string> strs;  // STRSXP payload
  std::vector<SEXPREC*> elems;    // VECSXP payload
  std::vector<std::string> names;
  bool has_dim = false;
  int nrow = 0;
  int ncol = 0;
  std::string s4_class;
  std::map<std::string, SEXPREC*> slots;
};
typedef SEXPREC* SEXP;
typedef std::ptrdiff_t R_xlen_t;

namespace rshim {

inline std::mutex& pool_mutex() {
  static std::mutex m;
  return m;
}
inline std::vector<std::unique_ptr<SEXPREC>>& pool() {
  static std::vector<std::unique_ptr<SEXPREC>> p;
  return p;
}
inline SEXP alloc(int type) {
  std::lock_guard<std::mutex> lock(pool_mutex());
  pool().emplace_back(new SEXPREC());
  SEXP s = pool().back().get();
  s->type = type;
  return s;
}
// Release every object created since the last collect().  Only safe when no
// Rcpp-typed value created before the call is still in use.
inline void collect() {
  std::lock_guard<std::mutex> lock(pool_mutex());
  pool().clear();
}
inline SEXP nil() {
  static SEXPREC n;
  return &n;
}
inline std::string& last_warning() {
  static std::string w;
  return w;
}
inline std::string vformat(const char* fmt, va_list ap) {
  char buf[2048];
  std::vsnprintf(buf, sizeof(buf), fmt, ap);
  return std::string(buf);
}

}  // namespace rshim

static const int NA_INTEGER = std::numeric_limits<int>::min();
static const double NA_REAL = std::numeric_limits<double>::quiet_NaN();
static const double R_NaReal = std::numeric_limits<double>::quiet_NaN();
static SEXPREC rshim_dim_symbol_storage;
static const SEXP R_DimSymbol = &rshim_dim_symbol_storage;

inline int TYPEOF(SEXP x) { return x == nullptr ? NILSXP : x->type; }
inline int* INTEGER(SEXP x) { return x->ints.data(); }
inline int* LOGICAL(SEXP x) { return x->ints.data(); }
inline double* REAL(SEXP x) { return x->reals.data(); }
inline bool Rf_isS4(SEXP x) { return x != nullptr && x->type == S4SXP; }
inline bool Rf_isNull(SEXP x) { return x == nullptr || x->type == NILSXP; }
inline bool Rf_isMatrix(SEXP x) { return x != nullptr && x->has_dim; }
inline bool Rf_isReal(SEXP x) { return x != nullptr && x->type == REALSXP; }
inline SEXP Rf_getAttrib(SEXP x, SEXP sym) {
  if (sym == R_DimSymbol && x != nullptr && x->has_dim) {
    SEXP d = rshim::alloc(INTSXP);
    d->ints = {x->nrow, x->ncol};
    return d;
  }
  return rshim::nil();
}
inline R_xlen_t Rf_xlength(SEXP x) {
  if (x == nullptr) return 0;
  switch (x->type) {
    case INTSXP:
    case LGLSXP: return static_cast<R_xlen_t>(x->ints.size());
    case REALSXP: return static_cast<R_xlen_t>(x->reals.size());
    case STRSXP: return static_cast<R_xlen_t>(x->strs.size());
    case VECSXP: return static_cast<R_xlen_t>(x->elems.size());
    default: return 0;
  }
}
inline R_xlen_t XLENGTH(SEXP x) { return Rf_xlength(x); }
inline int LENGTH(SEXP x) { return static_cast<int>(Rf_xlength(x)); }
inline int Rf_length(SEXP x) { return static_cast<int>(Rf_xlength(x)); }

namespace Rcpp {

[[noreturn]] inline void stop(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  std::string msg = rshim::vformat(fmt, ap);
  va_end(ap);
  throw std::runtime_error(msg);
}
[[noreturn]] inline void stop(const std::string& msg) { throw std::runtime_error(msg); }
inline void warning(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  rshim::last_warning() = rshim::vformat(fmt, ap);
  va_end(ap);
}
inline void warning(const std::string& msg) { rshim::last_warning() = msg; }
inline void checkUserInterrupt() {}

// Rcout: silent unless FE_ORACLE_VERBOSE is set.
struct NullBuffer : std::streambuf {
  int overflow(int c) override { return c; }
};
inline std::ostream& rcout_stream() {
  static NullBuffer nb;
  static std::ostream null_stream(&nb);
  return std::getenv("FE_ORACLE_VERBOSE") != nullptr ? std::cout : null_stream;
}
#define Rcout rcout_stream()

template <int RTYPE> struct storage;
template <> struct storage<INTSXP> { typedef int type; };
template <> struct storage<LGLSXP> { typedef int type; };
template <> struct storage<REALSXP> { typedef double type; };

template <int RTYPE> inline typename storage<RTYPE>::type* data_ptr(SEXP s);
template <> inline int* data_ptr<INTSXP>(SEXP s) { return s->ints.data(); }
template <> inline int* data_ptr<LGLSXP>(SEXP s) { return s->ints.data(); }
template <> inline double* data_ptr<REALSXP>(SEXP s) { return s->reals.data(); }

template <int RTYPE> inline void resize_payload(SEXP s, std::size_t n);
template <> inline void resize_payload<INTSXP>(SEXP s, std::size_t n) { s->ints.assign(n, 0); }
template <> inline void resize_payload<LGLSXP>(SEXP s, std::size_t n) { s->ints.assign(n, 0); }
template <> inline void resize_payload<REALSXP>(SEXP s, std::size_t n) { s->reals.assign(n, 0.0); }

inline SEXP coerce(SEXP x, int type) {
  if (x == nullptr || x->type == type) return x;
  SEXP out = rshim::alloc(type);
  out->has_dim = x->has_dim;
  out->nrow = x->nrow;
  out->ncol = x->ncol;
  if (type == REALSXP && (x->type == INTSXP || x->type == LGLSXP)) {
    out->reals.resize(x->ints.size());
    for (std::size_t i = 0; i < x->ints.size(); ++i) {
      out->reals[i] = x->ints[i] == NA_INTEGER ? NA_REAL : static_cast<double>(x->ints[i]);
    }
  } else if ((type == INTSXP || type == LGLSXP) && x->type == REALSXP) {
    out->ints.resize(x->reals.size());
    for (std::size_t i = 0; i < x->reals.size(); ++i) out->ints[i] = static_cast<int>(x->reals[i]);
  } else if ((type == INTSXP || type == LGLSXP) && (x->type == INTSXP || x->type == LGLSXP)) {
    out->ints = x->ints;
  } else {
    stop("rshim: unsupported coercion");
  }
  return out;
}

template <int RTYPE>
class Vector {
 public:
  typedef typename storage<RTYPE>::type value_type;
  typedef value_type* iterator;
  typedef const value_type* const_iterator;

  Vector() : s_(rshim::alloc(RTYPE)) {}
  explicit Vector(SEXP x) : s_(coerce(x, RTYPE)) {}
  template <typename IntT, typename = typename std::enable_if<std::is_integral<IntT>::value>::type>
  explicit Vector(IntT n) : s_(rshim::alloc(RTYPE)) { resize_payload<RTYPE>(s_, static_cast<std::size_t>(n)); }
  template <typename IntT, typename = typename std::enable_if<std::is_integral<IntT>::value>::type>
  Vector(IntT n, value_type fill) : s_(rshim::alloc(RTYPE)) {
    resize_payload<RTYPE>(s_, static_cast<std::size_t>(n));
    std::fill(begin(), end(), fill);
  }
  template <typename It, typename = typename std::enable_if<!std::is_integral<It>::value>::type>
  Vector(It first, It last) : s_(rshim::alloc(RTYPE)) {
    const std::size_t n = static_cast<std::size_t>(std::distance(first, last));
    resize_payload<RTYPE>(s_, n);
    value_type* p = data_ptr<RTYPE>(s_);
    for (std::size_t i = 0; first != last; ++first, ++i) p[i] = static_cast<value_type>(*first);
  }
  template <typename... Args>
  static Vector create(Args... args) {
    Vector v(static_cast<int>(sizeof...(Args)));
    value_type vals[] = {static_cast<value_type>(args)...};
    for (std::size_t i = 0; i < sizeof...(Args); ++i) v[static_cast<int>(i)] = vals[i];
    return v;
  }

  operator SEXP() const { return s_; }
  SEXP get__() const { return s_; }
  R_xlen_t size() const { return Rf_xlength(s_); }
  R_xlen_t length() const { return Rf_xlength(s_); }
  iterator begin() { return data_ptr<RTYPE>(s_); }
  iterator end() { return data_ptr<RTYPE>(s_) + size(); }
  const_iterator begin() const { return data_ptr<RTYPE>(s_); }
  const_iterator end() const { return data_ptr<RTYPE>(s_) + size(); }
  value_type& operator[](R_xlen_t i) { return data_ptr<RTYPE>(s_)[i]; }
  const value_type& operator[](R_xlen_t i) const { return data_ptr<RTYPE>(s_)[i]; }
  value_type& operator()(R_xlen_t i) { return data_ptr<RTYPE>(s_)[i]; }
  const value_type& operator()(R_xlen_t i) const { return data_ptr<RTYPE>(s_)[i]; }

 protected:
  SEXP s_;
};

template <int RTYPE>
class Matrix : public Vector<RTYPE> {
 public:
  typedef typename Vector<RTYPE>::value_type value_type;
  Matrix() : Vector<RTYPE>() { this->s_->has_dim = true; }
  explicit Matrix(SEXP x) : Vector<RTYPE>(x) {
    if (!this->s_->has_dim) {
      this->s_->has_dim = true;
      this->s_->nrow = static_cast<int>(Rf_xlength(this->s_));
      this->s_->ncol = 1;
    }
  }
  Matrix(int nrow, int ncol) : Vector<RTYPE>(static_cast<std::size_t>(nrow) * static_cast<std::size_t>(ncol)) {
    this->s_->has_dim = true;
    this->s_->nrow = nrow;
    this->s_->ncol = ncol;
  }
  int nrow() const { return this->s_->nrow; }
  int ncol() const { return this->s_->ncol; }
  int rows() const { return this->s_->nrow; }
  int cols() const { return this->s_->ncol; }
  value_type& operator()(int i, int j) {
    return data_ptr<RTYPE>(this->s_)[static_cast<std::size_t>(j) * this->s_->nrow + i];
  }
  const value_type& operator()(int i, int j) const {
    return data_ptr<RTYPE>(this->s_)[static_cast<std::size_t>(j) * this->s_->nrow + i];
  }
};

typedef Vector<INTSXP> IntegerVector;
typedef Vector<REALSXP> NumericVector;
typedef Vector<LGLSXP> LogicalVector;
typedef Matrix<INTSXP> IntegerMatrix;
typedef Matrix<REALSXP> NumericMatrix;

inline SEXP wrap(SEXP x) { return x; }
inline SEXP wrap(double v) {
  SEXP s = rshim::alloc(REALSXP);
  s->reals = {v};
  return s;
}
inline SEXP wrap(float v) { return wrap(static_cast<double>(v)); }
inline SEXP wrap(int v) {
  SEXP s = rshim::alloc(INTSXP);
  s->ints = {v};
  return s;
}
inline SEXP wrap(unsigned int v) { return wrap(static_cast<double>(v)); }
inline SEXP wrap(long v) { return wrap(static_cast<double>(v)); }
inline SEXP wrap(unsigned long v) { return wrap(static_cast<double>(v)); }
inline SEXP wrap(bool v) {
  SEXP s = rshim::alloc(LGLSXP);
  s->ints = {v ? 1 : 0};
  return s;
}
inline SEXP wrap(const std::string& v) {
  SEXP s = rshim::alloc(STRSXP);
  s->strs = {v};
  return s;
}
inline SEXP wrap(const char* v) { return wrap(std::string(v)); }
inline SEXP wrap(const std::vector<int>& v) {
  SEXP s = rshim::alloc(INTSXP);
  s->ints = v;
  return s;
}
inline SEXP wrap(const std::vector<double>& v) {
  SEXP s = rshim::alloc(REALSXP);
  s->reals = v;
  return s;
}
inline SEXP wrap(const std::vector<float>& v) {
  SEXP s = rshim::alloc(REALSXP);
  s->reals.assign(v.begin(), v.end());
  return s;
}
inline SEXP wrap(const std::vector<std::string>& v) {
  SEXP s = rshim::alloc(STRSXP);
  s->strs = v;
  return s;
}
template <int RTYPE>
inline SEXP wrap(const Vector<RTYPE>& v) { return v.get__(); }
template <int RTYPE>
inline SEXP wrap(const Matrix<RTYPE>& v) { return v.get__(); }

struct NamedArg {
  std::string name;
  SEXP value = nullptr;
  template <typename T>
  NamedArg& operator=(const T& v) {
    value = wrap(v);
    return *this;
  }
};
inline NamedArg Named(const std::string& name) {
  NamedArg a;
  a.name = name;
  return a;
}
template <typename T>
inline NamedArg Named(const std::string& name, const T& v) {
  NamedArg a;
  a.name = name;
  a.value = wrap(v);
  return a;
}

class List {
 public:
  List() : s_(rshim::alloc(VECSXP)) {}
  explicit List(SEXP x) : s_(x) {}
  template <typename... Args>
  static List create(const Args&... args) {
    List out;
    add(out, args...);
    return out;
  }
  operator SEXP() const { return s_; }
  R_xlen_t size() const { return Rf_xlength(s_); }
  SEXP operator[](const std::string& name) const {
    for (std::size_t i = 0; i < s_->names.size(); ++i) {
      if (s_->names[i] == name) return s_->elems[i];
    }
    return rshim::nil();
  }
  SEXP operator[](int i) const { return s_->elems[static_cast<std::size_t>(i)]; }

 private:
  static void add(List&) {}
  template <typename... Rest>
  static void add(List& out, const NamedArg& first, const Rest&... rest) {
    out.s_->elems.push_back(first.value);
    out.s_->names.push_back(first.name);
    add(out, rest...);
  }
  SEXP s_;
};

class S4 {
 public:
  explicit S4(SEXP x) : s_(x) {}
  bool is(const std::string& klass) const { return s_ != nullptr && s_->s4_class == klass; }
  struct SlotProxy {
    SEXP v;
    operator SEXP() const { return v; }
    template <int RTYPE>
    operator Matrix<RTYPE>() const { return Matrix<RTYPE>(v); }
    template <int RTYPE>
    operator Vector<RTYPE>() const { return Vector<RTYPE>(v); }
  };
  SlotProxy slot(const std::string& name) const {
    auto it = s_->slots.find(name);
    if (it == s_->slots.end()) stop("rshim: missing S4 slot");
    return SlotProxy{it->second};
  }

 private:
  SEXP s_;
};

template <int RTYPE>
inline Matrix<RTYPE> clone(const Matrix<RTYPE>& m) {
  Matrix<RTYPE> out(m.nrow(), m.ncol());
  std::copy(m.begin(), m.end(), out.begin());
  return out;
}
template <int RTYPE>
inline Vector<RTYPE> clone(const Vector<RTYPE>& v) {
  Vector<RTYPE> out(v.begin(), v.end());
  return out;
}

template <typename T>
inline T as(SEXP x);
template <>
inline double as<double>(SEXP x) {
  if (x->type == REALSXP) return x->reals.at(0);
  return static_cast<double>(x->ints.at(0));
}
template <>
inline int as<int>(SEXP x) {
  if (x->type == REALSXP) return static_cast<int>(x->reals.at(0));
  return x->ints.at(0);
}
template <>
inline std::string as<std::string>(SEXP x) { return x->strs.at(0); }

}  // namespace Rcpp

// Convenience constructors used by the harnesses.
namespace rshim {

inline Rcpp::IntegerMatrix int_matrix(const int* col_major, int nrow, int ncol) {
  Rcpp::IntegerMatrix m(nrow, ncol);
  std::memcpy(m.begin(), col_major, sizeof(int) * static_cast<std::size_t>(nrow) * ncol);
  return m;
}
inline Rcpp::NumericMatrix real_matrix(const double* col_major, int nrow, int ncol) {
  Rcpp::NumericMatrix m(nrow, ncol);
  std::memcpy(m.begin(), col_major, sizeof(double) * static_cast<std::size_t>(nrow) * ncol);
  return m;
}
// float32 S4 object (package `float`): integer matrix payload holding float bits.
inline SEXP float32_matrix(const float* col_major, int nrow, int ncol) {
  Rcpp::IntegerMatrix payload(nrow, ncol);
  std::memcpy(payload.begin(), col_major, sizeof(float) * static_cast<std::size_t>(nrow) * ncol);
  SEXP s = alloc(S4SXP);
  s->s4_class = "float32";
  s->slots["Data"] = payload;
  return s;
}
inline SEXP float32_vector(const float* values, int n) {
  Rcpp::IntegerVector payload(n);
  std::memcpy(payload.begin(), values, sizeof(float) * static_cast<std::size_t>(n));
  SEXP s = alloc(S4SXP);
  s->s4_class = "float32";
  s->slots["Data"] = payload;
  return s;
}

}  // namespace rshim
