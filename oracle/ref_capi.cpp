// Test infrastructure only (parity checker, never the product path).
//
// extern "C" entry points that run the REFERENCE's own CPU implementation
// (silarray include/array.h + include/cpu.h, compiled unmodified except for
// the mechanical g++-13 rewrite done by oracle/patch_ref.py) on caller
// buffers.  Every entry point switches the reference to Device::CPU
// (include/device.h:15) and goes through the public sil::array API, so the
// arithmetic is exactly what a reference user gets in CPU mode:
//   elementwise + broadcasting  include/array.h:1312-1335, 2478-2600; cpu.h:76-237
//   affine folding              include/array.h:1888-1940, 1989-2023
//   dot / linear / batched_dot  include/array.h:1359-1416, 2161-2226, 2632-2655
//   softmax (row-min variant)   include/array.h:2135-2150
//   layer_norm                  include/cpu.h:352-373
//   argmax (first index)        include/array.h:1711-1750
//   sum / sum(axis) / min / max include/array.h:1523-1658, 2275-2319
// Built by oracle/Makefile into oracle/_ref/libsilref.so.
#include <silarray.h>

#include <cstring>
#include <exception>
#include <vector>

using sil::array;
using sil::shape_type;

namespace {

template <class T>
array<T> make(const T *p, const size_t *shape, int ndim) {
  shape_type sh(shape, shape + ndim);
  size_t n = 1;
  for (auto d : sh) n *= d;
  return array<T>(sh, std::vector<T>(p, p + n));
}

template <class T>
size_t copy_out(const array<T> &a, T *out, size_t cap) {
  auto n = a.element_count();
  if (n > cap) return static_cast<size_t>(-1);
  for (size_t i = 0; i < n; i++) out[i] = a.at(i);
  return n;
}

thread_local char g_err[512];

template <class F>
int guarded(F f) {
  try {
    sil::use_cpu();
    f();
    return 0;
  } catch (const std::exception &e) {
    std::strncpy(g_err, e.what(), sizeof(g_err) - 1);
    return 1;
  }
}

}  // namespace

extern "C" {

const char *silref_last_error(void) { return g_err; }

// op: 0 add, 1 sub, 2 mul, 3 div, 4 pow.  Returns 0 on success, 1 when the
// reference throws (message via silref_last_error); *out_n = elements written.
int silref_binary_f32(int op, const float *a, const size_t *ash, int andim,
                      const float *b, const size_t *bsh, int bndim, float *out,
                      size_t cap, size_t *out_n) {
  return guarded([&] {
    auto A = make(a, ash, andim), B = make(b, bsh, bndim);
    array<float> C;
    switch (op) {
      case 0: C = A + B; break;
      case 1: C = A - B; break;
      case 2: C = A * B; break;
      case 3: C = A / B; break;
      default: C = A.pow(B); break;
    }
    sil::eval(C);
    *out_n = copy_out(C, out, cap);
  });
}

int silref_binary_i32(int op, const int *a, const size_t *ash, int andim,
                      const int *b, const size_t *bsh, int bndim, int *out,
                      size_t cap, size_t *out_n) {
  return guarded([&] {
    auto A = make(a, ash, andim), B = make(b, bsh, bndim);
    array<int> C;
    switch (op) {
      case 0: C = A + B; break;
      case 1: C = A - B; break;
      case 2: C = A * B; break;
      case 3: C = A / B; break;
      default: C = A.pow(B); break;
    }
    *out_n = copy_out(C, out, cap);
  });
}

// A chain of scalar operations applied lazily to x, then evaluated once, so
// that the reference's affine folding (include/array.h:1888-1940) runs.
// ops[i]: 0 add, 1 sub, 2 mul, 3 div; left[i] != 0 puts the scalar on the left.
int silref_scalar_chain_f32(const float *x, size_t n, const int *ops,
                            const float *scalars, const int *left, int nops,
                            float *out) {
  return guarded([&] {
    size_t sh[1] = {n};
    auto X = make(x, sh, 1);
    array<float> Y = X;
    for (int i = 0; i < nops; i++) {
      array<float> s(scalars[i]);
      if (left[i]) {
        switch (ops[i]) {
          case 0: Y = s + Y; break;
          case 1: Y = s - Y; break;
          case 2: Y = s * Y; break;
          default: Y = s / Y; break;
        }
      } else {
        switch (ops[i]) {
          case 0: Y = Y + s; break;
          case 1: Y = Y - s; break;
          case 2: Y = Y * s; break;
          default: Y = Y / s; break;
        }
      }
    }
    sil::eval(Y);
    copy_out(Y, out, n);
  });
}

// unary: 0 sigmoid, 1 relu
int silref_unary_f32(int op, const float *x, size_t n, float *out) {
  return guarded([&] {
    size_t sh[1] = {n};
    auto X = make(x, sh, 1);
    array<float> Y = op == 0 ? X.sigmoid() : X.relu();
    sil::eval(Y);
    copy_out(Y, out, n);
  });
}

int silref_sigmoid_backward_f32(const float *s, const float *dout, size_t n,
                                float *out) {
  return guarded([&] {
    size_t sh[1] = {n};
    auto S = make(s, sh, 1), D = make(dout, sh, 1);
    auto Y = S.sigmoid_backward(D);
    sil::eval(Y);
    copy_out(Y, out, n);
  });
}

// C[M,N] = op(A) . op(B); when tA, A is stored [K,M] and viewed transposed;
// when tB, B is stored [N,K].
int silref_dot_f32(const float *a, const float *b, float *c, size_t M,
                   size_t N, size_t K, int tA, int tB) {
  return guarded([&] {
    size_t ash[2] = {tA ? K : M, tA ? M : K};
    size_t bsh[2] = {tB ? N : K, tB ? K : N};
    auto A = make(a, ash, 2), B = make(b, bsh, 2);
    if (tA) A = A.transpose();
    if (tB) B = B.transpose();
    auto C = A.dot(B);
    sil::eval(C);
    copy_out(C, c, M * N);
  });
}

// The 1-D promotions of dot (include/array.h:2698-2728): ndim 1 or 2 each.
int silref_dot_nd_f32(const float *a, const size_t *ash, int andim,
                      const float *b, const size_t *bsh, int bndim, float *out,
                      size_t cap, size_t *out_n) {
  return guarded([&] {
    auto A = make(a, ash, andim), B = make(b, bsh, bndim);
    auto C = A.dot(B);
    sil::eval(C);
    *out_n = copy_out(C, out, cap);
  });
}

int silref_dot_i32(const int *a, const int *b, int *c, size_t M, size_t N,
                   size_t K) {
  return guarded([&] {
    size_t ash[2] = {M, K}, bsh[2] = {K, N};
    auto A = make(a, ash, 2), B = make(b, bsh, 2);
    auto C = A.dot(B);
    copy_out(C, c, M * N);
  });
}

// act: 0 linear, 1 linear_sigmoid.  bias has blen elements (broadcast).
int silref_linear_f32(int act, const float *x, const float *w, const float *b,
                      size_t blen, float *y, size_t M, size_t N, size_t K) {
  return guarded([&] {
    size_t xsh[2] = {M, K}, wsh[2] = {K, N}, bsh[1] = {blen};
    auto X = make(x, xsh, 2), W = make(w, wsh, 2), B = make(b, bsh, 1);
    auto Y = act ? X.linear_sigmoid(W, B) : X.linear(W, B);
    sil::eval(Y);
    copy_out(Y, y, M * N);
  });
}

int silref_batched_dot_f32(const float *a, const float *b, float *c,
                           size_t batch, size_t M, size_t N, size_t K) {
  return guarded([&] {
    size_t ash[3] = {batch, M, K}, bsh[3] = {batch, K, N};
    auto A = make(a, ash, 3), B = make(b, bsh, 3);
    auto C = A.batched_dot(B);
    sil::eval(C);
    copy_out(C, c, batch * M * N);
  });
}

int silref_softmax_f32(const float *x, float *y, size_t rows, size_t cols) {
  return guarded([&] {
    size_t sh[2] = {rows, cols};
    auto X = make(x, sh, 2);
    auto Y = X.softmax();
    sil::eval(Y);
    copy_out(Y, y, rows * cols);
  });
}

int silref_softmax1d_f32(const float *x, float *y, size_t n) {
  return guarded([&] {
    size_t sh[1] = {n};
    auto X = make(x, sh, 1);
    auto Y = X.softmax();
    sil::eval(Y);
    copy_out(Y, y, n);
  });
}

int silref_layer_norm_f32(const float *x, const float *g, const float *b,
                          float *y, size_t rows, size_t cols, float eps) {
  return guarded([&] {
    size_t sh[2] = {rows, cols}, vsh[1] = {cols};
    auto X = make(x, sh, 2), G = make(g, vsh, 1), B = make(b, vsh, 1);
    auto Y = X.layer_norm(G, B, eps);
    sil::eval(Y);
    copy_out(Y, y, rows * cols);
  });
}

int silref_argmax_f32(const float *x, int *idx, size_t rows, size_t cols) {
  return guarded([&] {
    size_t sh[2] = {rows, cols};
    auto X = make(x, sh, 2);
    auto I = X.argmax();
    copy_out(I, idx, rows);
  });
}

int silref_argmax_i32(const int *x, int *idx, size_t rows, size_t cols) {
  return guarded([&] {
    size_t sh[2] = {rows, cols};
    auto X = make(x, sh, 2);
    auto I = X.argmax();
    copy_out(I, idx, rows);
  });
}

int silref_sum_axis_f32(const float *x, const size_t *sh, int ndim,
                        size_t axis, float *out, size_t cap, size_t *out_n) {
  return guarded([&] {
    auto X = make(x, sh, ndim);
    auto Y = X.sum(axis);
    sil::eval(Y);
    *out_n = copy_out(Y, out, cap);
  });
}

int silref_sum_axis_i32(const int *x, const size_t *sh, int ndim, size_t axis,
                        int *out, size_t cap, size_t *out_n) {
  return guarded([&] {
    auto X = make(x, sh, ndim);
    auto Y = X.sum(axis);
    *out_n = copy_out(Y, out, cap);
  });
}

// which: 0 sum, 1 min, 2 max
int silref_reduce_f32(int which, const float *x, size_t n, float *out) {
  return guarded([&] {
    size_t sh[1] = {n};
    auto X = make(x, sh, 1);
    *out = which == 0 ? X.sum() : which == 1 ? X.min() : X.max();
  });
}

int silref_reduce_i32(int which, const int *x, size_t n, int *out) {
  return guarded([&] {
    size_t sh[1] = {n};
    auto X = make(x, sh, 1);
    *out = which == 0 ? X.sum() : which == 1 ? X.min() : X.max();
  });
}

// Pre-norm transformer block (the graph of bench/composite/bench_transformer.cpp:56-67)
// generalised to `batch` sequences and `heads` heads of width d/heads, built
// only from reference ops.  Per-head column slices of Q/K/V are copied into
// their own arrays (data movement only; the reference API has no column view).
// x, out: [batch*seq, d].  W1: [d, dff], W2: [dff, d].
int silref_transformer_block_f32(const float *x, size_t batch, size_t seq,
                                 size_t d, size_t heads, size_t dff,
                                 const float *g1, const float *be1,
                                 const float *wq, const float *bq,
                                 const float *wk, const float *bk,
                                 const float *wv, const float *bv,
                                 const float *wo, const float *bo,
                                 const float *g2, const float *be2,
                                 const float *w1, const float *b1,
                                 const float *w2, const float *b2, float *out) {
  return guarded([&] {
    size_t dd[2] = {d, d}, d1[1] = {d}, dfs[2] = {d, dff}, fds[2] = {dff, d},
           f1[1] = {dff};
    auto G1 = make(g1, d1, 1), BE1 = make(be1, d1, 1);
    auto G2 = make(g2, d1, 1), BE2 = make(be2, d1, 1);
    auto WQ = make(wq, dd, 2), WK = make(wk, dd, 2), WV = make(wv, dd, 2),
         WO = make(wo, dd, 2);
    auto BQ = make(bq, d1, 1), BK = make(bk, d1, 1), BV = make(bv, d1, 1),
         BO = make(bo, d1, 1);
    auto W1 = make(w1, dfs, 2), B1 = make(b1, f1, 1);
    auto W2 = make(w2, fds, 2), B2 = make(b2, d1, 1);
    const size_t hd = d / heads;
    const float scale = 1.0f / std::sqrt(static_cast<float>(hd));
    for (size_t bi = 0; bi < batch; bi++) {
      size_t xs[2] = {seq, d};
      auto X = make(x + bi * seq * d, xs, 2);
      auto h = X.layer_norm(G1, BE1);
      auto Q = h.linear(WQ, BQ);
      auto K = h.linear(WK, BK);
      auto V = h.linear(WV, BV);
      sil::eval(Q, K, V);
      std::vector<float> ctx(seq * d);
      for (size_t hh = 0; hh < heads; hh++) {
        std::vector<float> q(seq * hd), k(seq * hd), v(seq * hd);
        for (size_t r = 0; r < seq; r++)
          for (size_t c = 0; c < hd; c++) {
            q[r * hd + c] = Q[r, hh * hd + c];
            k[r * hd + c] = K[r, hh * hd + c];
            v[r * hd + c] = V[r, hh * hd + c];
          }
        shape_type hs{seq, hd};
        array<float> Qh(hs, q), Kh(hs, k), Vh(hs, v);
        auto scores = Qh.dot(Kh.transpose()) * scale;
        auto attn = scores.softmax();
        auto c = attn.dot(Vh);
        sil::eval(c);
        for (size_t r = 0; r < seq; r++)
          for (size_t cc = 0; cc < hd; cc++)
            ctx[r * d + hh * hd + cc] = c[r, cc];
      }
      array<float> C(shape_type{seq, d}, ctx);
      auto attn_out = C.linear(WO, BO);
      auto r1 = X + attn_out;
      auto h2 = r1.layer_norm(G2, BE2);
      auto ff = h2.linear(W1, B1).relu();
      auto o = r1 + ff.linear(W2, B2);
      sil::eval(o);
      copy_out(o, out + bi * seq * d, seq * d);
    }
  });
}

}  // extern "C"
