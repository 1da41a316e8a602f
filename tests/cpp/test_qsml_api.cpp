// The qsml:: / QuasarML::Ops API on the B200 backend, checked the way the
// reference's unit tests check it (a pass/fail counter, nonzero exit on any
// failure): the known answers of unit-tests/src/_test_comprehensive.cpp,
// _test_qsml_functionality.cpp and _test_minimal.cpp, then the ops this
// backend adds (broadcasting, pow, axis max/min, argmax/argmin, strided
// slices, layer norm, batched and fp16 matmul, concat/stack, deferred fused
// elementwise results) and the error convention.
#include <QuasarML.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <iostream>
#include <stdexcept>
#include <vector>

using std::vector;

static int passed = 0, failed = 0;

static void check(const char* name, bool ok) {
    if (ok) {
        ++passed;
    } else {
        ++failed;
        std::cout << "FAIL: " << name << "\n";
    }
}

static vector<float> get(const qsml::TensorPtr& t) {
    vector<float> v(t->numel());
    t->download(v.data(), v.size() * sizeof(float));
    return v;
}

static bool near(float a, float b, float tol) { return std::fabs(a - b) < tol; }

static void test_device() {
    check("device_count >= 1", qsml::device_count() >= 1);
    check("device_names not empty", !qsml::device_names().empty());
    check("device is_valid", qsml::device().is_valid());
    check("current_device_id valid", qsml::current_device_id() < qsml::device_count());
}

static void test_creation() {
    auto z = qsml::zeros({16, 16});
    check("zeros shape", z->dim(0) == 16 && z->dim(1) == 16 && z->numel() == 256 && z->rank() == 2);
    bool all_zero = true;
    for (float v : get(z)) all_zero &= v == 0.0f;
    check("zeros values", all_zero);
    auto o = qsml::ones({8});
    bool all_one = true;
    for (float v : get(o)) all_one &= v == 1.0f;
    check("ones values", all_one);
    vector<float> input = {1, 2, 3, 4, 5, 6};
    auto t = qsml::from_data(input.data(), {2, 3}, qsml::DataType::F32);
    auto out = get(t);
    check("from_data roundtrip", out[0] == 1.0f && out[5] == 6.0f);
    auto two = get(qsml::add(qsml::ones({2, 2}), qsml::ones({2, 2})));
    check("ones + ones = 2", near(two[0], 2.0f, 1e-4f));
}

static void test_elementwise() {
    vector<float> a_data = {1, 2, 3, 4}, b_data = {5, 6, 7, 8}, c_data = {10, 20, 30, 40};
    auto a = qsml::from_data(a_data.data(), {4});
    auto b = qsml::from_data(b_data.data(), {4});
    auto c = qsml::from_data(c_data.data(), {4});
    auto s = get(qsml::add(a, b));
    check("add", near(s[0], 6, 1e-5f) && near(s[3], 12, 1e-5f));
    check("sub", near(get(qsml::sub(b, a))[0], 4, 1e-5f));
    check("mul", near(get(qsml::mul(a, b))[0], 5, 1e-5f));
    check("div", near(get(qsml::div(b, a))[0], 5, 1e-5f));
    check("neg", near(get(qsml::neg(a))[0], -1, 1e-5f));
    check("abs", near(get(qsml::abs(qsml::neg(a)))[0], 1, 1e-5f));
    check("mul_scalar x10", near(get(qsml::mul_scalar(a, 10.0f))[0], 10, 1e-5f));
    auto s2 = get(qsml::add(a, c));
    check("add (functionality)", near(s2[0], 11, 1e-5f) && near(s2[3], 44, 1e-5f));
    check("sub (functionality)", near(get(qsml::sub(c, a))[0], 9, 1e-5f));
    check("div (functionality)", near(get(qsml::div(c, a))[0], 10, 1e-5f));
    check("mul_scalar x2", near(get(qsml::mul_scalar(a, 2.0f))[0], 2, 1e-5f));
}

static void test_unary_and_activations() {
    vector<float> d = {0.25f, 1.0f, 4.0f, 9.0f};
    auto sq = get(qsml::sqrt(qsml::from_data(d.data(), {4})));
    check("sqrt", near(sq[0], 0.5f, 1e-4f) && near(sq[2], 2.0f, 1e-4f));
    vector<float> e = {0.0f, 1.0f, 2.0f};
    check("exp at 0", near(get(qsml::exp(qsml::from_data(e.data(), {3})))[0], 1.0f, 1e-4f));
    vector<float> x = {-1.0f, 0.0f, 1.0f, 2.0f};
    auto t = qsml::from_data(x.data(), {4});
    auto r = get(qsml::relu(t));
    check("relu negatives zeroed", r[0] == 0.0f);
    check("relu positives preserved", r[2] == 1.0f);
    check("sigmoid at 0 = 0.5", near(get(qsml::sigmoid(t))[1], 0.5f, 1e-4f));
    check("gelu computed", get(qsml::gelu(t))[2] > 0.5f);
    check("tanh at 0 = 0", near(get(qsml::tanh(t))[1], 0.0f, 1e-4f));
}

static void test_matrix() {
    auto c = qsml::matmul(qsml::ones({2, 3}), qsml::ones({3, 4}));
    check("matmul shape", c->dim(0) == 2 && c->dim(1) == 4);
    check("matmul values (inner dim 3)", near(get(c)[0], 3.0f, 1e-4f));
    auto tt = qsml::transpose(qsml::ones({4, 5}));
    check("transpose shape", tt->dim(0) == 5 && tt->dim(1) == 4);
}

static void test_reductions() {
    vector<float> d = {1, 2, 3, 4, 5, 6, 7, 8, 9, 10};
    auto a = qsml::from_data(d.data(), {10});
    check("sum", near(get(qsml::sum(a))[0], 55.0f, 1e-3f));
    check("mean", near(get(qsml::mean(a))[0], 5.5f, 1e-3f));
    check("max", near(get(qsml::max(a))[0], 10.0f, 1e-3f));
    check("min", near(get(qsml::min(a))[0], 1.0f, 1e-3f));
    check("prod of 1..10", near(get(qsml::prod(a))[0], 3628800.0f, 1.0f));
}

static void test_shapes() {
    auto a = qsml::ones({2, 3, 4});
    check("original shape", a->dim(0) == 2 && a->dim(1) == 3 && a->dim(2) == 4);
    auto f = qsml::flatten(a);
    check("flatten", f->numel() == 24 && f->rank() == 1);
    auto r = qsml::reshape(a, {6, 4});
    check("reshape", r->dim(0) == 6 && r->dim(1) == 4);
    auto s = qsml::squeeze(qsml::ones({1, 4, 1}));
    check("squeeze", s->rank() == 1 && s->numel() == 4);
    auto u = qsml::unsqueeze(qsml::ones({4}), 0);
    check("unsqueeze", u->rank() == 2 && u->dim(0) == 1);
}

static void test_broadcast_pow() {
    vector<float> m = {1, 2, 3, 4, 5, 6}, row = {10, 20, 30}, col = {100, 200};
    auto A = qsml::from_data(m.data(), {2, 3});
    auto r = get(qsml::add(A, qsml::from_data(row.data(), {3})));
    check("broadcast row", r[0] == 11 && r[5] == 36);
    auto c = get(qsml::mul(A, qsml::from_data(col.data(), {2, 1})));
    check("broadcast column", c[0] == 100 && c[5] == 1200);
    auto p = get(qsml::pow(A, 2.0f));
    check("pow x^2 exact", p[2] == 9.0f && p[5] == 36.0f);
    vector<float> e = {0.5f, 1.0f, 3.0f};
    auto pe = get(qsml::pow(A, qsml::from_data(e.data(), {3})));
    check("pow tensor exponent", near(pe[0], 1.0f, 1e-6f) && near(pe[2], 27.0f, 1e-4f) && near(pe[3], 2.0f, 1e-6f));
}

static void test_axis_reductions() {
    vector<float> m = {1, 9, 3, 7, 5, 2};  // [[1,9,3],[7,5,2]]
    auto A = qsml::from_data(m.data(), {2, 3});
    auto mx0 = get(qsml::max(A, 0));
    check("max axis 0", mx0.size() == 3 && mx0[0] == 7 && mx0[1] == 9 && mx0[2] == 3);
    auto mn1 = get(qsml::min(A, 1));
    check("min axis 1", mn1.size() == 2 && mn1[0] == 1 && mn1[1] == 2);
    auto s1 = qsml::sum(A, -1, true);
    check("sum keepdims shape", s1->rank() == 2 && s1->dim(0) == 2 && s1->dim(1) == 1);
    auto sv = get(s1);
    check("sum axis 1", sv[0] == 13 && sv[1] == 14);
    check("mean axis 0", get(qsml::mean(A, 0))[1] == 7.0f);
    // argmax/argmin give I32 indices (the reference's stubs return max/min values)
    auto am = qsml::argmax(A);  // last axis
    vector<int32_t> ai(am->numel());
    am->download(ai.data(), ai.size() * sizeof(int32_t));
    check("argmax dtype/shape", am->dtype() == QuasarML::DataType::I32 && am->rank() == 1 && am->dim(0) == 2);
    check("argmax axis -1", ai[0] == 1 && ai[1] == 0);
    auto an = qsml::argmin(A, 0);
    vector<int32_t> ni(an->numel());
    an->download(ni.data(), ni.size() * sizeof(int32_t));
    check("argmin axis 0", ni.size() == 3 && ni[0] == 0 && ni[1] == 1 && ni[2] == 1);
}

static void test_views_and_gathers() {
    vector<float> v(8 * 6);
    for (size_t i = 0; i < v.size(); ++i) v[i] = static_cast<float>(i);
    auto X = qsml::from_data(v.data(), {8, 6});
    auto s = qsml::slice(qsml::slice(X, 0, 1, 8, 3), 1, 1, 6, 2);  // X[1::3, 1::2]
    check("slice shape", s->dim(0) == 3 && s->dim(1) == 3 && !s->is_contiguous());
    auto sv = get(s);
    check("slice values", sv[0] == 7 && sv[1] == 9 && sv[3] == 25 && sv[8] == 47);
    auto T = qsml::transpose(X, 0, 1);
    check("transpose is a view", !T->is_contiguous() && T->storage() == X->storage());
    auto tc = get(qsml::contiguous(T));
    check("transpose values", tc[1] == 6 && tc[8] == 1);
    auto ts = get(qsml::slice(T, 0, 0, 6, 4));  // X.T[::4, :]
    check("strided transpose slice", ts.size() == 16 && ts[0] == 0 && ts[8] == 4 && ts[9] == 10);
    // reductions of views read the view in place (no contiguous copy)
    auto ss = get(qsml::sum(s, 1));  // rows of X[1::3, 1::2]: 7+9+11, 25+27+29, 43+45+47
    check("sum over a sliced view", ss.size() == 3 && ss[0] == 27 && ss[1] == 81 && ss[2] == 135);
    auto st0 = get(qsml::sum(T, 1));  // X.T summed over its columns = X's row sums
    check("sum over a transposed view", st0.size() == 6 && st0[0] == 0 + 6 + 12 + 18 + 24 + 30 + 36 + 42);
    check("max of a sliced view", get(qsml::max(s))[0] == 47 && get(qsml::min(s))[0] == 7);
    check("mean of a transposed view", near(get(qsml::mean(T))[0], 23.5f, 1e-5f));
    // independent reductions give the same results with overlap on (the
    // default) and off
    for (bool ov : {true, false}) {
        qsml::set_overlap(ov);
        auto o1 = qsml::sum(X, 1), o2 = qsml::max(X, 0), o3 = qsml::sum(s, 1), o4 = qsml::sum(o1);
        auto v1 = get(o1), v2 = get(o2), v3 = get(o3), v4 = get(o4);
        check(ov ? "overlapped reductions" : "reductions without overlap",
              v1[0] == 15 && v1[7] == 42 * 6 + 15 && v2[5] == 47 && v3[1] == 81 && v4[0] == 47.0f * 48.0f / 2.0f);
    }
    qsml::set_overlap(true);
    // argmax over an axis of a transpose reads it in place; of a slice, a copy
    auto idx = [](const qsml::TensorPtr& t) {
        vector<int32_t> v(t->numel());
        t->download(v.data(), v.size() * sizeof(int32_t));
        return v;
    };
    auto amv = idx(qsml::argmax(T, 1));  // X.T [6, 8]: each row's largest is X's last row
    check("argmax over a transposed view", amv.size() == 6 && amv[0] == 7 && amv[5] == 7);
    auto as = idx(qsml::argmin(s, 0));  // X[1::3, 1::2] [3, 3]: the first row is smallest
    check("argmin over a sliced view", as.size() == 3 && as[0] == 0 && as[2] == 0);
    auto cat = qsml::concat({X, X}, 1);
    auto cv = get(cat);
    check("concat axis 1", cat->dim(1) == 12 && cv[6] == 0 && cv[13] == 7);
    auto st = qsml::stack({qsml::ones({2, 2}), qsml::zeros({2, 2})}, 0);
    auto stv = get(st);
    check("stack", st->dim(0) == 2 && stv[0] == 1 && stv[4] == 0);
    auto bt = get(qsml::broadcast_to(qsml::from_data(v.data(), {1, 3}), {4, 3}));
    check("broadcast_to", bt[9] == 0 && bt[11] == 2);
    auto sm = get(qsml::sum(qsml::softmax(X, -1), -1));
    bool ones = true;
    for (float x : sm) ones &= near(x, 1.0f, 1e-5f);
    check("softmax rows sum to 1", ones);
}

static void test_layer_norm_and_matmul() {
    const unsigned R = 4, C = 64;
    vector<float> x(R * C), g(C, 1.0f), b(C, 0.0f);
    for (size_t i = 0; i < x.size(); ++i) x[i] = std::sin(0.37f * i) * 3.0f + 1.0f;
    auto y = get(qsml::layer_norm(qsml::from_data(x.data(), {R, C}), qsml::from_data(g.data(), {C}),
                                  qsml::from_data(b.data(), {C}), 1e-5f));
    bool ok = true;
    for (unsigned r = 0; r < R; ++r) {
        double m = 0, v = 0;
        for (unsigned c = 0; c < C; ++c) m += y[r * C + c];
        m /= C;
        for (unsigned c = 0; c < C; ++c) v += (y[r * C + c] - m) * (y[r * C + c] - m);
        v /= C;
        ok &= std::fabs(m) < 1e-5 && std::fabs(v - 1.0) < 1e-3;
    }
    check("layer_norm rows have mean 0, variance 1", ok);

    const unsigned B = 3, M = 5, K = 7, N = 4;
    vector<float> a(B * M * K), w(B * K * N);
    for (size_t i = 0; i < a.size(); ++i) a[i] = std::cos(0.1f * i);
    for (size_t i = 0; i < w.size(); ++i) w[i] = std::sin(0.2f * i);
    auto At = qsml::from_data(a.data(), {B, M, K});
    auto Wt = qsml::from_data(w.data(), {B, K, N});
    auto Cb = get(qsml::batch_matmul(At, Wt));
    bool bm = true;
    for (unsigned i = 0; i < B; ++i) {
        auto Ci = get(qsml::matmul(qsml::from_data(a.data() + i * M * K, {M, K}),
                                   qsml::from_data(w.data() + i * K * N, {K, N})));
        for (unsigned j = 0; j < M * N; ++j) bm &= Ci[j] == Cb[i * M * N + j];
    }
    check("batch_matmul equals per-slice matmul", bm);

    // fp16 inputs on the tensor cores, fp32 result, against the fp32 product
    const unsigned S = 256;
    vector<float> p(S * S), q(S * S);
    for (size_t i = 0; i < p.size(); ++i) {
        p[i] = std::sin(0.013f * i) * 0.25f;
        q[i] = std::cos(0.007f * i) * 0.25f;
    }
    vector<uint16_t> ph(S * S), qh(S * S);
    auto to_half = [](float f) {  // values here are normal binary16 numbers
        uint32_t x;
        std::memcpy(&x, &f, 4);
        uint32_t sign = (x >> 16) & 0x8000u, e = (x >> 23) & 0xffu, man = x & 0x7fffffu;
        if (e == 0) return static_cast<uint16_t>(sign);
        int he = static_cast<int>(e) - 127 + 15;
        if (he <= 0) return static_cast<uint16_t>(sign);
        uint32_t h = (static_cast<uint32_t>(he) << 10) | (man >> 13), rem = man & 0x1fffu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
        return static_cast<uint16_t>(sign | h);
    };
    for (size_t i = 0; i < p.size(); ++i) {
        ph[i] = to_half(p[i]);
        qh[i] = to_half(q[i]);
    }
    auto Ch = get(qsml::matmul(qsml::from_data(ph.data(), {S, S}, qsml::DataType::F16),
                               qsml::from_data(qh.data(), {S, S}, qsml::DataType::F16), qsml::DataType::F32));
    auto Cf = get(qsml::matmul(qsml::from_data(p.data(), {S, S}), qsml::from_data(q.data(), {S, S})));
    double err = 0, ref = 0;
    for (size_t i = 0; i < Ch.size(); ++i) {
        err = std::max(err, static_cast<double>(std::fabs(Ch[i] - Cf[i])));
        ref = std::max(ref, static_cast<double>(std::fabs(Cf[i])));
    }
    check("fp16 tensor-core matmul within 1e-2 of fp32", err / ref < 1e-2);
}

static uint64_t launches() {
    uint64_t n = 0;
    qsml::device().check(qsml_launch_count(qsml::device().ctx(), &n));
    return n;
}

static bool same_bits(const vector<float>& a, const vector<float>& b) {
    return a.size() == b.size() && std::memcmp(a.data(), b.data(), a.size() * sizeof(float)) == 0;
}

// Deferred elementwise results (set_fusion / begin_batch): one fused launch,
// bit-identical to eager execution, writes after deferred reads, long chains.
static void test_fusion() {
    const qsml::u32 R = 64, C = 256;
    vector<float> a(R * C), b(C), dv(R);
    uint32_t x = 12345u;
    auto rnd = [&](float lo, float hi) {
        x = x * 1664525u + 1013904223u;
        return lo + (hi - lo) * static_cast<float>(x >> 8) / 16777216.0f;
    };
    for (auto& v : a) v = rnd(-1, 1);
    for (auto& v : b) v = rnd(-1, 1);
    for (auto& v : dv) v = rnd(0.5f, 2.0f);
    auto A = qsml::from_data(a.data(), {R, C});
    auto B = qsml::from_data(b.data(), {1, C});
    auto D = qsml::from_data(dv.data(), {R, 1});
    auto chain = [&]() {
        return qsml::relu(qsml::div(qsml::pow(qsml::sub(qsml::mul(qsml::add(A, B), B), A), 2.0f), D));
    };
    auto eager = get(chain());
    qsml::set_fusion(true);
    const uint64_t l0 = launches();
    auto T = chain();
    check("fusion: result deferred", T->is_lazy() && launches() == l0);
    auto fused = get(T);
    check("fusion: one launch for the chain", launches() - l0 == 1);
    check("fusion: bit-identical to eager", same_bits(eager, fused));

    // a write into an input evaluates the deferred readers first
    qsml::set_fusion(false);
    auto ref_sum = get(qsml::add(A, B));
    qsml::set_fusion(true);
    auto U = qsml::add(A, B);
    vector<float> zeros(R * C, 0.0f);
    A->upload(zeros.data());
    check("fusion: deferred read before a write sees old data", same_bits(get(U), ref_sum));
    A->upload(a.data());

    // a chain longer than one fused kernel takes splits itself
    qsml::TensorPtr L = A;
    for (int i = 0; i < 100; ++i) L = qsml::add_scalar(L, 0.25f);
    auto long_fused = get(L);
    qsml::set_fusion(false);
    qsml::TensorPtr E = A;
    for (int i = 0; i < 100; ++i) E = qsml::add_scalar(E, 0.25f);
    check("fusion: 100-op chain equals eager", same_bits(long_fused, get(E)));

    // the reference's batch bracket defers too
    qsml::device().begin_batch();
    auto Tb = chain();
    qsml::device().end_batch();
    check("batch: deferred inside begin/end_batch", Tb->is_lazy());
    check("batch: bit-identical to eager", same_bits(get(Tb), eager));
    check("fusion off again", !qsml::fusion_enabled());
}

// All-reduce across the devices of this process (identity with one GPU).
static void test_all_reduce() {
    const qsml::u32 n = qsml::device_count() >= 2 ? 2 : 1;
    std::vector<qsml::TensorPtr> parts;
    for (qsml::u32 i = 0; i < n; ++i) {
        vector<float> v(1024, static_cast<float>(i + 1));
        auto t = qsml::device(i).create_tensor({1024});
        t->upload(v.data());
        parts.push_back(t);
    }
    qsml::all_reduce(parts, qsml::ReduceOp::Sum);
    const float want = n == 2 ? 3.0f : 1.0f;
    bool ok = true;
    for (auto& t : parts) {
        auto v = get(t);
        ok &= v[0] == want && v[1023] == want;
    }
    check("all_reduce sum across devices", ok);
    qsml::all_reduce(parts, qsml::ReduceOp::Max);
    check("all_reduce max", get(parts[0])[5] == want);
}

static void test_errors_and_counters() {
    bool threw = false;
    try {
        qsml::add(qsml::ones({3, 4}), qsml::ones({5}));
    } catch (const std::runtime_error&) {
        threw = true;
    }
    check("shape mismatch throws std::runtime_error", threw);
    threw = false;
    try {
        qsml::matmul(qsml::ones({2, 3}), qsml::ones({4, 5}));
    } catch (const std::runtime_error&) {
        threw = true;
    }
    check("matmul inner mismatch throws", threw);
    qsml::synchronize();
    check("cpu_fallback_count == 0", qsml::cpu_fallback_count() == 0);
}

// Row-sharded reductions over as many devices as there are (two at most):
// results equal the host's reduction of the whole tensor; -0 and +0 in one
// column must give +0 for max and -0 for min across the blocks.
static void test_sharded_reduce() {
    const unsigned R = 10, C = 6;
    vector<float> v(R * C);
    for (size_t i = 0; i < v.size(); ++i) v[i] = std::sin(0.7f * i) * 3.0f;
    for (unsigned r = 0; r < R; ++r) v[r * C + 4] = (r % 2) ? 0.0f : -0.0f;
    const unsigned nd = std::min(2u, qsml::device_count());
    auto blocks = qsml::scatter_rows(v.data(), {R, C}, nd);
    check("scatter_rows blocks", blocks.size() == nd && blocks[0]->dim(0) == (nd == 2 ? 5 : 10));
    auto cs = qsml::sharded_reduce(blocks, qsml::ReduceOp::Sum, 0);
    auto mx = qsml::sharded_reduce(blocks, qsml::ReduceOp::Max, 0);
    auto mn = qsml::sharded_reduce(blocks, qsml::ReduceOp::Min, 0);
    auto all = qsml::sharded_reduce(blocks, qsml::ReduceOp::Mean);
    bool ok_sum = true, ok_max = true, ok_min = true, ok_mean = true;
    double total = 0;
    for (float x : v) total += x;
    for (unsigned d = 0; d < nd; ++d) {
        auto s = get(cs[d]), m = get(mx[d]), n = get(mn[d]), a = get(all[d]);
        for (unsigned c = 0; c < C; ++c) {
            double want = 0;
            float hi = -INFINITY, lo = INFINITY;
            for (unsigned r = 0; r < R; ++r) {
                want += v[r * C + c];
                hi = std::max(hi, v[r * C + c]);
                lo = std::min(lo, v[r * C + c]);
            }
            ok_sum &= near(s[c], static_cast<float>(want), 1e-4f);
            if (c == 4) {
                ok_max &= m[c] == 0.0f && !std::signbit(m[c]);
                ok_min &= n[c] == 0.0f && std::signbit(n[c]);
            } else {
                ok_max &= m[c] == hi;
                ok_min &= n[c] == lo;
            }
        }
        ok_mean &= a.size() == 1 && near(a[0], static_cast<float>(total / (R * C)), 1e-5f);
    }
    check("sharded sum over rows", ok_sum);
    check("sharded max over rows (+0 beats -0)", ok_max);
    check("sharded min over rows (-0 beats +0)", ok_min);
    check("sharded mean of all elements", ok_mean);
    auto rm = qsml::sharded_reduce(blocks, qsml::ReduceOp::Mean, 1);
    auto r0 = get(rm[0]);
    double row0 = 0;
    for (unsigned c = 0; c < C; ++c) row0 += v[c];
    check("sharded mean over columns stays row-local", rm[0]->dim(0) == blocks[0]->dim(0) &&
                                                           near(r0[0], static_cast<float>(row0 / C), 1e-5f));
}

int main() {
    qsml::init();
    try {
        test_device();
        test_creation();
        test_elementwise();
        test_unary_and_activations();
        test_matrix();
        test_reductions();
        test_shapes();
        test_broadcast_pow();
        test_axis_reductions();
        test_views_and_gathers();
        test_layer_norm_and_matmul();
        test_fusion();
        test_all_reduce();
        test_sharded_reduce();
        test_errors_and_counters();
    } catch (const std::exception& e) {
        std::cout << "EXCEPTION: " << e.what() << "\n";
        ++failed;
    }
    std::cout << "passed " << passed << ", failed " << failed << "\n";
    qsml::shutdown();
    return failed == 0 ? 0 : 1;
}
