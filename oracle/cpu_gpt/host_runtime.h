// TEST INFRASTRUCTURE: a complete host runtime for TempLit's typed executor
// (satisfies passes::Runnable), restating every op of the reference's Metal
// runtime in C++ on the CPU:
//   elementwise / broadcast ops   math.metal:401-548, runtime.cpp:18-39,65-136
//   mult (batched, broadcast)     runtime.cpp:375-505 (infer_shape.h:65-112)
//   transpose                     runtime.cpp:529-569, math.metal:566-584
//   sum / sum_to_shape / max      runtime.cpp:506-527,595-745, math.metal:549-714
//   softmax, cross-entropy (+')   runtime.cpp:747-841, math.metal:857-953
//   RMS, RMSNorm                  runtime.cpp:1031-1072
//   GELU, GELU'                   math.metal:821-855
//   embedding gather / scatter    runtime.cpp:920-1030, math.metal:778-820
//   norm, clip, AdamW             runtime.cpp:1083-1168, math.metal:955-1043
// Reductions and products accumulate in double.  It drives the reference's
// own passes::Compiled (the GPT step oracle and the CPU baseline); the
// product never links it.  OpenMP parallelises the outer loops.
#pragma once

#include "RTensor/RTensor.h"
#include "RTensor/dimension.h"
#include "RTensor/infer_shape.h"
#include "RTensor/storage.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <numeric>
#include <span>
#include <stdexcept>
#include <vector>

namespace cpu_ref {
struct Host {};
using kernel_type = float;
using index_type = uint32_t;
}  // namespace cpu_ref

template <typename T> class Storage<cpu_ref::Host, T> {
public:
  explicit Storage(size_t n) : ref_count(1), data_(n) {}
  int ref_count;
  T *data() { return data_.data(); }
  const T *data() const { return data_.data(); }
  size_t size() const { return data_.size(); }
  void write(std::span<const T> v, size_t off) {
    if (off + v.size() > data_.size()) throw std::out_of_range("write out of bounds");
    std::copy(v.begin(), v.end(), data_.begin() + off);
  }
  void read(std::span<T> out, size_t off) const {
    if (off + out.size() > data_.size()) throw std::out_of_range("read out of bounds");
    std::copy(data_.begin() + off, data_.begin() + off + out.size(), out.begin());
  }
  void fill(T v) { std::fill(data_.begin(), data_.end(), v); }
  Storage *clone() const {
    auto *o = new Storage(data_.size());
    o->data_ = data_;
    return o;
  }
  bool compare(const Storage &o) const { return data_ == o.data_; }

private:
  std::vector<T> data_;
};

namespace cpu_ref {

using Mat = RTensor<Host, float>;
using IMat = RTensor<Host, uint32_t>;

inline const float *P(const Mat &m) { return m.get_storage()->data(); }
inline float *P(Mat &m) { return m.get_storage()->data(); }

// strides of `shape` broadcast (trailing-aligned) against `out`
inline std::vector<size_t> bstrides(const std::vector<uint32_t> &shape,
                                    const std::vector<uint32_t> &out) {
  if (shape.size() > out.size()) throw std::runtime_error("invalid broadcast");
  std::vector<size_t> dense(shape.size()), r(out.size(), 0);
  size_t s = 1;
  for (size_t i = shape.size(); i-- > 0;) {
    dense[i] = s;
    s *= shape[i];
  }
  const size_t off = out.size() - shape.size();
  for (size_t i = 0; i < shape.size(); ++i) {
    if (shape[i] == out[off + i]) r[off + i] = dense[i];
    else if (shape[i] == 1) r[off + i] = 0;
    else throw std::runtime_error("invalid broadcast");
  }
  return r;
}

class Runtime {
public:
  // Data parallelism, as the CUDA runtime's optimiser windows do it: every
  // gradient an optimiser op reads is first summed across ranks, once per
  // window (the callback performs the sum in place).
  using AllReduceFn = void (*)(float *data, uint64_t count, void *ctx);
  AllReduceFn allreduce = nullptr;
  void *allreduce_ctx = nullptr;
  std::vector<const void *> reduced;  // gradients summed in this window

  void start() { reduced.clear(); }
  void submit() {}
  void wait() {}

  void reduce_once(const Mat &g) {
    if (!allreduce) return;
    const void *key = g.get_storage()->data();
    for (const void *k : reduced)
      if (k == key) return;
    reduced.push_back(key);
    allreduce(const_cast<float *>(P(g)), g.numel(), allreduce_ctx);
  }
  void abort() noexcept {}
  void cleanup() noexcept {}

  template <typename F>
  void binary(const Mat &a, const Mat &b, Mat &o, F f) {
    const auto &os = o.shape();
    const auto sa = bstrides(a.shape(), os), sb = bstrides(b.shape(), os);
    const size_t n = o.numel(), r = os.size();
    std::vector<size_t> ost(r);
    size_t s = 1;
    for (size_t i = r; i-- > 0;) {
      ost[i] = s;
      s *= os[i];
    }
    const float *pa = P(a), *pb = P(b);
    // out may alias an input element for element: stage the result
    std::vector<float> tmp(n);
#pragma omp parallel for schedule(static)
    for (size_t e = 0; e < n; ++e) {
      size_t rem = e, ia = 0, ib = 0;
      for (size_t d = 0; d < r; ++d) {
        const size_t c = rem / ost[d];
        rem -= c * ost[d];
        ia += c * sa[d];
        ib += c * sb[d];
      }
      tmp[e] = f(pa[ia], pb[ib]);
    }
    std::copy(tmp.begin(), tmp.end(), P(o));
  }
  template <typename F> void unary(const Mat &a, Mat &o, F f) {
    if (a.numel() != o.numel()) throw std::invalid_argument("unary size mismatch");
    const float *pa = P(a);
    float *po = P(o);
    const size_t n = o.numel();
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; ++i) po[i] = f(pa[i]);
  }
  void scalar_check(const Mat &a, const Mat &o) {
    if (a.shape() != o.shape())
      throw std::invalid_argument("scalar operation input and output shapes must match");
  }

  void add(const Mat &a, const Mat &b, Mat &o) { binary(a, b, o, [](float x, float y) { return x + y; }); }
  void sub(const Mat &a, const Mat &b, Mat &o) { binary(a, b, o, [](float x, float y) { return x - y; }); }
  void hadamard(const Mat &a, const Mat &b, Mat &o) { binary(a, b, o, [](float x, float y) { return x * y; }); }
  void divide(const Mat &a, const Mat &b, Mat &o) { binary(a, b, o, [](float x, float y) { return x / y; }); }
  void add(const Mat &a, float s, Mat &o) { scalar_check(a, o); unary(a, o, [s](float x) { return x + s; }); }
  void divide(const Mat &a, float s, Mat &o) { scalar_check(a, o); unary(a, o, [s](float x) { return x / s; }); }
  void pow(const Mat &a, float s, Mat &o) {
    scalar_check(a, o);
    unary(a, o, [s](float x) { return static_cast<float>(std::pow(double(x), double(s))); });
  }
  void sigmoid(const Mat &a, Mat &o) {
    unary(a, o, [](float x) { return static_cast<float>(1.0 / (1.0 + std::exp(-double(x)))); });
  }
  void sqrt(const Mat &a, Mat &o) { unary(a, o, [](float x) { return static_cast<float>(std::sqrt(double(x))); }); }
  void exp(const Mat &a, Mat &o) { unary(a, o, [](float x) { return static_cast<float>(std::exp(double(x))); }); }
  static double gelu(double x) {
    const double k = std::sqrt(2.0 / 3.14159265);
    return 0.5 * x * (1.0 + std::tanh(k * (x + 0.044715 * x * x * x)));
  }
  static double gelu_d(double x) {
    const double a = 0.7978845608, b = 0.044715;
    const double t = std::tanh(a * (x + b * x * x * x));
    return 0.5 * (1.0 + t) + 0.5 * x * (1.0 - t * t) * a * (1.0 + 3.0 * b * x * x);
  }
  void GELU(const Mat &a, Mat &o) { unary(a, o, [](float x) { return float(gelu(x)); }); }
  void GELU_derivative(const Mat &a, Mat &o) { unary(a, o, [](float x) { return float(gelu_d(x)); }); }
  void copy(const Mat &a, Mat &o) {
    if (a.shape() != o.shape()) throw std::invalid_argument("copy destination has incorrect shape");
    std::copy(P(a), P(a) + a.numel(), P(o));
  }
  void sqe(const Mat &p, const Mat &t, Mat &o) {
    sub(p, t, o);
    hadamard(o, o, o);
  }

  void mult(const Mat &a, const Mat &b, Mat &o) {
    const auto expect = rtensor::infer_mult(a.shape(), b.shape());
    if (o.shape() != expect) throw std::invalid_argument("matmul destination has incorrect shape");
    const auto &as = a.shape(), &bs = b.shape(), &cs = o.shape();
    const size_t M = as[as.size() - 2], K = as.back(), N = bs.back();
    const size_t br = cs.size() - 2;
    std::vector<uint32_t> cb(cs.begin(), cs.end() - 2);
    auto batch_strides = [&](const std::vector<uint32_t> &sh, size_t mat) {
      std::vector<uint32_t> b_(sh.begin(), sh.end() - 2);
      std::vector<size_t> st(br, 0);
      size_t acc = mat;
      const size_t off = br - b_.size();
      for (size_t i = b_.size(); i-- > 0;) {
        st[off + i] = b_[i] == 1 ? 0 : acc;
        acc *= b_[i];
      }
      return st;
    };
    const auto sa = batch_strides(as, M * K), sb = batch_strides(bs, K * N);
    size_t batches = 1;
    for (auto d : cb) batches *= d;
    const float *pa = P(a), *pb = P(b);
    float *pc = P(o);
#pragma omp parallel for schedule(dynamic, 1) collapse(2)
    for (size_t z = 0; z < batches; ++z) {
      for (size_t i = 0; i < M; ++i) {
        size_t rem = z, oa = 0, ob = 0;
        for (size_t d = br; d-- > 0;) {
          const size_t c = rem % cb[d];
          rem /= cb[d];
          oa += c * sa[d];
          ob += c * sb[d];
        }
        std::vector<double> acc(N, 0.0);
        const float *ar = pa + oa + i * K;
        for (size_t k = 0; k < K; ++k) {
          const double av = ar[k];
          const float *brow = pb + ob + k * N;
          for (size_t j = 0; j < N; ++j) acc[j] += av * brow[j];
        }
        float *cr = pc + z * M * N + i * N;
        for (size_t j = 0; j < N; ++j) cr[j] = static_cast<float>(acc[j]);
      }
    }
  }

  void transpose(const Mat &a, Mat &o, int32_t da = -2, int32_t db = -1) {
    if (a.shape().size() < 2) throw std::invalid_argument("transpose requires rank >= 2");
    const size_t x = rtensor::normalise_dimension(a.shape().size(), da);
    const size_t y = rtensor::normalise_dimension(a.shape().size(), db);
    if (x == y) throw std::invalid_argument("transpose dimensions must be different");
    if (o.shape() != rtensor::infer_transpose(a.shape(), da, db))
      throw std::invalid_argument("transpose destination has incorrect shape");
    auto ist = a.strides();
    std::swap(ist[x], ist[y]);
    const auto &ost = o.strides();
    const size_t n = o.numel(), r = ost.size();
    const float *pa = P(a);
    float *po = P(o);
#pragma omp parallel for schedule(static)
    for (size_t e = 0; e < n; ++e) {
      size_t rem = e, off = 0;
      for (size_t d = 0; d < r; ++d) {
        const size_t c = rem / ost[d];
        rem %= ost[d];
        off += c * ist[d];
      }
      po[e] = pa[off];
    }
  }
  void split_last_dim(const Mat &a, Mat &o, uint32_t outer, uint32_t inner) {
    if (o.shape() != rtensor::infer_split_last_dim(a.shape(), outer, inner))
      throw std::invalid_argument("split_last_dim destination has incorrect shape");
    std::copy(P(a), P(a) + a.numel(), P(o));
  }
  void merge_last_dims(const Mat &a, Mat &o, uint32_t outer, uint32_t inner) {
    if (o.shape() != rtensor::infer_merge_last_dims(a.shape(), outer, inner))
      throw std::invalid_argument("merge_last_dims destination has incorrect shape");
    std::copy(P(a), P(a) + a.numel(), P(o));
  }

  // out[o] = reduce over the dims where the trailing-aligned out shape is 1
  template <typename F>
  void reduce(const Mat &a, std::span<const uint32_t> oshape, Mat &o, double init, F f) {
    const auto &as = a.shape();
    if (oshape.size() > as.size())
      throw std::invalid_argument("cannot reduce to a shape with a higher rank");
    const size_t r = as.size(), off = r - oshape.size();
    std::vector<uint32_t> al(r, 1);
    for (size_t i = 0; i < oshape.size(); ++i) al[off + i] = oshape[i];
    for (size_t i = 0; i < r; ++i)
      if (as[i] != al[i] && al[i] != 1) throw std::invalid_argument("invalid reduce_to_shape");
    size_t outn = 1;
    for (auto d : al) outn *= d;
    std::vector<size_t> ost(r);
    size_t s = 1;
    for (size_t i = r; i-- > 0;) {
      ost[i] = al[i] == 1 ? 0 : s;
      s *= al[i];
    }
    std::vector<double> acc(outn, init);
    const size_t n = a.numel();
    const float *pa = P(a);
    const auto &ist = a.strides();
    // deterministic serial accumulation in input order
    for (size_t e = 0; e < n; ++e) {
      size_t rem = e, oi = 0;
      for (size_t d = 0; d < r; ++d) {
        const size_t c = rem / ist[d];
        rem %= ist[d];
        oi += c * ost[d];
      }
      acc[oi] = f(acc[oi], double(pa[e]));
    }
    float *po = P(o);
    for (size_t i = 0; i < outn; ++i) po[i] = static_cast<float>(acc[i]);
  }
  void sum(const Mat &a, Mat &o) {
    double t = 0;
    const float *pa = P(a);
    for (size_t i = 0; i < a.numel(); ++i) t += pa[i];
    P(o)[0] = static_cast<float>(t);
  }
  void sum(const Mat &a, size_t axis, Mat &o) {
    if (axis >= a.shape().size()) throw std::out_of_range("sum axis out of range");
    sum_to_shape(a, o.shape(), o);
  }
  void sum_to_shape(const Mat &a, std::span<const uint32_t> s, Mat &o) {
    if (o.shape().size() != s.size() || !std::equal(s.begin(), s.end(), o.shape().begin()))
      throw std::invalid_argument("sum_to_shape destination has incorrect shape");
    reduce(a, s, o, 0.0, [](double x, double y) { return x + y; });
  }
  void max_to_shape(const Mat &a, std::span<const uint32_t> s, Mat &o) {
    if (s.size() != a.shape().size()) throw std::invalid_argument("cannot reduce to shape if ranks differ");
    reduce(a, s, o, -std::numeric_limits<double>::infinity(),
           [](double x, double y) { return std::max(x, y); });
  }

  void softmax(const Mat &x, Mat &o) {
    if (x.shape().empty() || x.shape().back() == 0)
      throw std::invalid_argument("softmax requires a non-empty final dimension");
    if (o.shape() != x.shape()) throw std::invalid_argument("softmax destination has incorrect shape");
    const size_t c = x.shape().back(), rows = x.numel() / c;
    const float *px = P(x);
    float *po = P(o);
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < rows; ++r) {
      const float *xr = px + r * c;
      double m = -std::numeric_limits<double>::infinity(), s = 0;
      for (size_t j = 0; j < c; ++j) m = std::max(m, double(xr[j]));
      for (size_t j = 0; j < c; ++j) s += std::exp(double(xr[j]) - m);
      for (size_t j = 0; j < c; ++j) po[r * c + j] = static_cast<float>(std::exp(double(xr[j]) - m) / s);
    }
  }
  void xent_check(const Mat &z, const IMat &t) {
    if (z.shape().size() < 2 || z.shape().back() == 0)
      throw std::invalid_argument("cross_entropy requires logits with a non-empty final dimension");
    if (t.shape().size() + 1 != z.shape().size())
      throw std::invalid_argument("cross_entropy target rank must be one less than logits rank");
  }
  void cross_entropy(const Mat &z, const IMat &t, Mat &o) {
    xent_check(z, t);
    const size_t v = z.shape().back(), rows = t.numel();
    const float *pz = P(z);
    const uint32_t *pt = t.get_storage()->data();
    float *po = P(o);
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < rows; ++r) {
      if (pt[r] >= v) {
        po[r] = std::numeric_limits<float>::infinity();
        continue;
      }
      const float *zr = pz + r * v;
      double m = -std::numeric_limits<double>::infinity(), s = 0;
      for (size_t j = 0; j < v; ++j) m = std::max(m, double(zr[j]));
      for (size_t j = 0; j < v; ++j) s += std::exp(double(zr[j]) - m);
      po[r] = static_cast<float>(m + std::log(s) - zr[pt[r]]);
    }
  }
  void cross_entropy_derivative(const Mat &z, const IMat &t, Mat &o) {
    xent_check(z, t);
    const size_t v = z.shape().back(), rows = t.numel();
    const float *pz = P(z);
    const uint32_t *pt = t.get_storage()->data();
    float *po = P(o);
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < rows; ++r) {
      float *orow = po + r * v;
      if (pt[r] >= v) {
        for (size_t j = 0; j < v; ++j) orow[j] = std::numeric_limits<float>::infinity();
        continue;
      }
      const float *zr = pz + r * v;
      double m = -std::numeric_limits<double>::infinity(), s = 0;
      for (size_t j = 0; j < v; ++j) m = std::max(m, double(zr[j]));
      for (size_t j = 0; j < v; ++j) s += std::exp(double(zr[j]) - m);
      for (size_t j = 0; j < v; ++j) {
        double p = std::exp(double(zr[j]) - m) / s;
        if (j == pt[r]) p -= 1.0;
        orow[j] = static_cast<float>(p);
      }
    }
  }
  void argmax(const Mat &a, IMat &o) {
    const float *pa = P(a);
    uint32_t best = 0;
    float bv = -std::numeric_limits<float>::infinity();
    for (size_t i = 0; i < a.numel(); ++i)
      if (pa[i] > bv) {
        bv = pa[i];
        best = static_cast<uint32_t>(i);
      }
    o.get_storage()->data()[0] = best;
  }
  void RMS(const Mat &x, Mat &o) {
    const size_t c = x.shape().back(), rows = x.numel() / c;
    const float *px = P(x);
    float *po = P(o);
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < rows; ++r) {
      double ss = 0;
      for (size_t j = 0; j < c; ++j) ss += double(px[r * c + j]) * px[r * c + j];
      po[r] = static_cast<float>(std::sqrt(ss / double(c) + 1e-6));
    }
  }
  void RMSNorm(const Mat &x, Mat &o) {
    const size_t c = x.shape().back(), rows = x.numel() / c;
    const float *px = P(x);
    float *po = P(o);
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < rows; ++r) {
      double ss = 0;
      for (size_t j = 0; j < c; ++j) ss += double(px[r * c + j]) * px[r * c + j];
      const double rms = std::sqrt(ss / double(c) + 1e-6);
      for (size_t j = 0; j < c; ++j) po[r * c + j] = static_cast<float>(px[r * c + j] / rms);
    }
  }
  void embedding_lookup(const Mat &w, const IMat &ids, Mat &o) {
    if (w.shape().size() != 2) throw std::invalid_argument("embedding weights must have rank 2");
    const size_t d = w.shape()[1], n = ids.numel(), rows = w.shape()[0];
    const uint32_t *pi = ids.get_storage()->data();
    for (size_t i = 0; i < n; ++i) {
      if (pi[i] >= rows) throw std::out_of_range("embedding id out of range");
      std::copy(P(w) + pi[i] * d, P(w) + (pi[i] + 1) * d, P(o) + i * d);
    }
  }
  void gather_rows(const Mat &w, const IMat &ids, Mat &o) { embedding_lookup(w, ids, o); }
  void scatter(const Mat &values, const IMat &ids, Mat &dst, const Mat *base) {
    const size_t d = dst.shape()[1], n = ids.numel(), rows = dst.shape()[0];
    std::vector<double> acc(rows * d, 0.0);
    const uint32_t *pi = ids.get_storage()->data();
    const float *pv = P(values);
    for (size_t i = 0; i < n; ++i) {
      if (pi[i] >= rows) throw std::out_of_range("scatter id out of range");
      for (size_t j = 0; j < d; ++j) acc[pi[i] * d + j] += pv[i * d + j];
    }
    float *po = P(dst);
    const float *pb = base ? P(*base) : nullptr;
    for (size_t e = 0; e < rows * d; ++e) po[e] = static_cast<float>((pb ? pb[e] : 0.0) + acc[e]);
  }
  void scatter_add_rows(const Mat &base, const IMat &ids, const Mat &values, Mat &dst) {
    if (base.shape() != dst.shape())
      throw std::invalid_argument("scatter base and destination shapes must match");
    scatter(values, ids, dst, &base);
  }
  void scatter_index(const Mat &values, const IMat &ids, Mat &dst) { scatter(values, ids, dst, nullptr); }
  void accumulate_gradient_squared_norm(const Mat &g, Mat &sq) {
    reduce_once(g);
    double s = 0;
    for (size_t i = 0; i < g.numel(); ++i) s += double(P(g)[i]) * P(g)[i];
    P(sq)[0] = static_cast<float>(double(P(sq)[0]) + s);
  }
  void clip_gradient(const Mat &g, const Mat &sq, float max_norm, Mat &o) {
    reduce_once(g);
    const double n2 = std::max(double(P(sq)[0]), 1e-12);
    const double sc = std::min(1.0, double(max_norm) / std::sqrt(n2));
    for (size_t i = 0; i < g.numel(); ++i) P(o)[i] = static_cast<float>(P(g)[i] * sc);
  }
  void adamW(const Mat &p, const Mat &g, Mat &o, Mat &m1, Mat &m2, const Mat &b1, const Mat &b2,
             const Mat &decay, const Mat &lr, float eps, uint32_t step) {
    if (step == 0) throw std::invalid_argument("AdamW step must be greater than zero");
    reduce_once(g);
    const double B1 = P(b1)[0], B2 = P(b2)[0], D = P(decay)[0], L = P(lr)[0];
    const double c1 = 1.0 - std::pow(B1, double(step)), c2 = 1.0 - std::pow(B2, double(step));
    const size_t n = p.numel();
    const float *pp = P(p), *pg = P(g);
    float *po = P(o), *pm = P(m1), *pv = P(m2);
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; ++i) {
      const double m = B1 * pm[i] + (1.0 - B1) * pg[i];
      const double v = B2 * pv[i] + (1.0 - B2) * double(pg[i]) * pg[i];
      pm[i] = static_cast<float>(m);
      pv[i] = static_cast<float>(v);
      po[i] = static_cast<float>(pp[i] * D - L * (m / c1) / (std::sqrt(v / c2) + eps));
    }
  }
};

}  // namespace cpu_ref
