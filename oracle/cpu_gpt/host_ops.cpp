// TEST INFRASTRUCTURE: the ops of the host oracle runtime (host_runtime.h)
// one by one behind a C ABI, so tests can pin them directly against the
// reference's known answers and the float64 restatement (oracle/ops.py)
// before the oracle is trusted as the GPT-step reference.  Every entry
// builds RTensor<Host, float> operands of the given shapes, calls the
// cpu_ref::Runtime method the reference executor calls, and copies the
// result out.  Returns 0, or -1 with the exception text in tlo_h_error().
#include "host_runtime.h"

#include <cstring>
#include <string>

namespace {

thread_local std::string g_err;

using cpu_ref::IMat;
using cpu_ref::Mat;

Mat make(const float *data, const uint32_t *shape, int rank) {
  Mat m(std::span<const uint32_t>(shape, static_cast<size_t>(rank)));
  if (data) std::memcpy(cpu_ref::P(m), data, m.numel() * sizeof(float));
  return m;
}

IMat make_ids(const uint32_t *data, const uint32_t *shape, int rank) {
  IMat m(std::span<const uint32_t>(shape, static_cast<size_t>(rank)));
  std::memcpy(m.get_storage()->data(), data, m.numel() * sizeof(uint32_t));
  return m;
}

void put(const Mat &m, float *out) {
  std::memcpy(out, cpu_ref::P(m), m.numel() * sizeof(float));
}

template <typename F> int guarded(F &&f) {
  try {
    f();
    return 0;
  } catch (const std::exception &e) {
    g_err = e.what();
  } catch (...) {
    g_err = "unknown exception";
  }
  return -1;
}

}  // namespace

extern "C" {

const char *tlo_h_error(void) { return g_err.c_str(); }

// add / sub / hadamard / divide with broadcasting (runtime.cpp:18-39)
int tlo_h_binary(const char *kind, const float *a, const uint32_t *as, int ar, const float *b,
                 const uint32_t *bs, int br, float *out, const uint32_t *os, int orank) {
  return guarded([&] {
    cpu_ref::Runtime rt;
    Mat A = make(a, as, ar), B = make(b, bs, br), O = make(nullptr, os, orank);
    const std::string k(kind);
    if (k == "add") rt.add(A, B, O);
    else if (k == "sub") rt.sub(A, B, O);
    else if (k == "mul") rt.hadamard(A, B, O);
    else if (k == "div") rt.divide(A, B, O);
    else throw std::invalid_argument("unknown binary op " + k);
    put(O, out);
  });
}

// x + s, x / s, x ^ s
int tlo_h_scalar(const char *kind, const float *x, uint32_t n, float s, float *out) {
  return guarded([&] {
    cpu_ref::Runtime rt;
    Mat X = make(x, &n, 1), O = make(nullptr, &n, 1);
    const std::string k(kind);
    if (k == "add") rt.add(X, s, O);
    else if (k == "div") rt.divide(X, s, O);
    else if (k == "pow") rt.pow(X, s, O);
    else throw std::invalid_argument("unknown scalar op " + k);
    put(O, out);
  });
}

// sigmoid / exp / sqrt / gelu / gelu_derivative
int tlo_h_unary(const char *kind, const float *x, uint32_t n, float *out) {
  return guarded([&] {
    cpu_ref::Runtime rt;
    Mat X = make(x, &n, 1), O = make(nullptr, &n, 1);
    const std::string k(kind);
    if (k == "sigmoid") rt.sigmoid(X, O);
    else if (k == "exp") rt.exp(X, O);
    else if (k == "sqrt") rt.sqrt(X, O);
    else if (k == "gelu") rt.GELU(X, O);
    else if (k == "gelu_derivative") rt.GELU_derivative(X, O);
    else throw std::invalid_argument("unknown unary op " + k);
    put(O, out);
  });
}

// batched / broadcast matrix product (runtime.cpp:375-505)
int tlo_h_mult(const float *a, const uint32_t *as, int ar, const float *b, const uint32_t *bs,
               int br, float *out, const uint32_t *os, int orank) {
  return guarded([&] {
    cpu_ref::Runtime rt;
    Mat A = make(a, as, ar), B = make(b, bs, br), O = make(nullptr, os, orank);
    rt.mult(A, B, O);
    put(O, out);
  });
}

int tlo_h_transpose(const float *x, const uint32_t *xs, int xr, int32_t da, int32_t db,
                    float *out, const uint32_t *os) {
  return guarded([&] {
    cpu_ref::Runtime rt;
    Mat X = make(x, xs, xr), O = make(nullptr, os, xr);
    rt.transpose(X, O, da, db);
    put(O, out);
  });
}

// sum_to_shape / max_to_shape (runtime.cpp:595-745)
int tlo_h_reduce(const char *kind, const float *x, const uint32_t *xs, int xr, float *out,
                 const uint32_t *os, int orank) {
  return guarded([&] {
    cpu_ref::Runtime rt;
    Mat X = make(x, xs, xr), O = make(nullptr, os, orank);
    const std::span<const uint32_t> s(os, static_cast<size_t>(orank));
    const std::string k(kind);
    if (k == "sum_to_shape") rt.sum_to_shape(X, s, O);
    else if (k == "max_to_shape") rt.max_to_shape(X, s, O);
    else throw std::invalid_argument("unknown reduction " + k);
    put(O, out);
  });
}

// row ops over the last dim: softmax (x -> same shape), rmsnorm (same
// shape), rms (one value per row: out shape = x shape with last dim 1)
int tlo_h_rows(const char *kind, const float *x, const uint32_t *xs, int xr, float *out,
               const uint32_t *os, int orank) {
  return guarded([&] {
    cpu_ref::Runtime rt;
    Mat X = make(x, xs, xr), O = make(nullptr, os, orank);
    const std::string k(kind);
    if (k == "softmax") rt.softmax(X, O);
    else if (k == "rmsnorm") rt.RMSNorm(X, O);
    else if (k == "rms") rt.RMS(X, O);
    else throw std::invalid_argument("unknown row op " + k);
    put(O, out);
  });
}

// cross_entropy (loss per row, out shape = z shape with last dim 1) or its
// derivative (z's shape); targets have z's shape without the last dim
int tlo_h_xent(int derivative, const float *z, const uint32_t *zs, int zr, const uint32_t *t,
               float *out, const uint32_t *os, int orank) {
  return guarded([&] {
    cpu_ref::Runtime rt;
    Mat Z = make(z, zs, zr), O = make(nullptr, os, orank);
    IMat T = make_ids(t, zs, zr - 1);
    if (derivative) rt.cross_entropy_derivative(Z, T, O);
    else rt.cross_entropy(Z, T, O);
    put(O, out);
  });
}

int tlo_h_argmax(const float *x, uint32_t n, uint32_t *out) {
  return guarded([&] {
    cpu_ref::Runtime rt;
    Mat X = make(x, &n, 1);
    const uint32_t one = 1;
    IMat O(std::span<const uint32_t>(&one, 1));
    rt.argmax(X, O);
    *out = O.get_storage()->data()[0];
  });
}

// out[i, :] = w[ids[i], :]
int tlo_h_gather(const float *w, uint32_t rows, uint32_t dim, const uint32_t *ids, uint32_t n,
                 float *out) {
  return guarded([&] {
    cpu_ref::Runtime rt;
    const uint32_t ws[2] = {rows, dim}, os[2] = {n, dim};
    Mat W = make(w, ws, 2), O = make(nullptr, os, 2);
    IMat I = make_ids(ids, &n, 1);
    rt.embedding_lookup(W, I, O);
    put(O, out);
  });
}

// dst = (base or 0) + values[i, :] summed into row ids[i]
int tlo_h_scatter(const float *values, const uint32_t *ids, uint32_t n, uint32_t dim,
                  const float *base, float *dst, uint32_t rows) {
  return guarded([&] {
    cpu_ref::Runtime rt;
    const uint32_t vs[2] = {n, dim}, ds[2] = {rows, dim};
    Mat V = make(values, vs, 2), D = make(nullptr, ds, 2);
    IMat I = make_ids(ids, &n, 1);
    if (base) {
      Mat B = make(base, ds, 2);
      rt.scatter_add_rows(B, I, V, D);
    } else {
      rt.scatter_index(V, I, D);
    }
    put(D, dst);
  });
}

// sqnorm += sum(g^2) for each of the n_tensors gradients, then each is
// clipped to max_norm (runtime.cpp:1083-1131)
int tlo_h_clip(const float *const *grads, const uint32_t *counts, int n_tensors,
               float max_norm, float *sqnorm, float *const *clipped) {
  return guarded([&] {
    cpu_ref::Runtime rt;
    const uint32_t one = 1;
    Mat SQ = make(nullptr, &one, 1);
    cpu_ref::P(SQ)[0] = 0.0f;
    std::vector<Mat> gs;
    for (int i = 0; i < n_tensors; ++i) gs.push_back(make(grads[i], &counts[i], 1));
    for (const Mat &g : gs) rt.accumulate_gradient_squared_norm(g, SQ);
    *sqnorm = cpu_ref::P(SQ)[0];
    for (int i = 0; i < n_tensors; ++i) {
      Mat O = make(nullptr, &counts[i], 1);
      rt.clip_gradient(gs[i], SQ, max_norm, O);
      put(O, clipped[i]);
    }
  });
}

// one AdamW step in place on p, m1, m2 (runtime.cpp:1132-1168)
int tlo_h_adamw(float *p, const float *g, float *m1, float *m2, uint32_t n, float beta1,
                float beta2, float decay, float lr, float eps, uint32_t step) {
  return guarded([&] {
    cpu_ref::Runtime rt;
    const uint32_t one = 1;
    Mat P = make(p, &n, 1), G = make(g, &n, 1), O = make(nullptr, &n, 1);
    Mat M1 = make(m1, &n, 1), M2 = make(m2, &n, 1);
    Mat B1 = make(&beta1, &one, 1), B2 = make(&beta2, &one, 1);
    Mat D = make(&decay, &one, 1), L = make(&lr, &one, 1);
    rt.adamW(P, G, O, M1, M2, B1, B2, D, L, eps, step);
    put(O, p);
    put(M1, m1);
    put(M2, m2);
  });
}

}  // extern "C"
