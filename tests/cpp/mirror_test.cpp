// Exercises the C++ host mirror (include/kernix_b200.hpp) the way Kernix's own
// tests exercise the Rust API.  `--host` needs no GPU; `--gpu` runs on device 0.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <utility>
#include <vector>

#include "kernix_b200.hpp"

static int failures = 0;
#define EXPECT(c)                                                        \
    do {                                                                 \
        if (!(c)) {                                                      \
            std::fprintf(stderr, "FAIL %s:%d: %s\n", __FILE__, __LINE__, #c); \
            ++failures;                                                  \
        }                                                                \
    } while (0)

static void host_checks() {
    // native_kernel_tests.rs:17-28: invalid span rejected, isize::MIN singleton accepted
    double one = 1.0;
    bool threw = false;
    try {
        kernix::MatrixInput<double>::create(&one, 1, {2, 2}, {2, 1}, 0);
    } catch (const kernix::OpsError &e) {
        threw = e.status() == KX_E_LAYOUT;
    }
    EXPECT(threw);
    auto m = kernix::MatrixInput<double>::create(&one, 1, {1, 1}, {INT64_MIN, INT64_MIN}, 0);
    EXPECT(m.strides()[0] == 0 && m.strides()[1] == 0);
    // ops_tests.rs:304-320: contraction mismatch carries (left, right)
    uint64_t a[2] = {2, 3}, b[2] = {4, 2}, od[KX_MAX_RANK];
    uint32_t r = 0;
    kx_error e{};
    EXPECT(kx_matmul_shape(a, 2, b, 2, &r, od, &e) == KX_E_CONTRACT && e.values[0] == 3 && e.values[1] == 4);
    // small_matmul_tests.rs:137-151: malformed extents decline without writes
    std::vector<float> out(64, 7.0f), x(16, 1.0f), y(63, 2.0f);
    EXPECT(kx_try_dense_matmul_f32(nullptr, x.data(), 16, y.data(), 63, out.data(), 64, 4, 4, 16) == KX_DECLINED);
    for (float v : out) EXPECT(v == 7.0f);
    // the [cuda] table is validated key by key before any device work
    kernix::CudaConfig bad;
    bad.c.f32_variant = 9;
    threw = false;
    try {
        kernix::Handle h(bad);
    } catch (const kernix::OpsError &e) {
        threw = e.status() == KX_E_PARAM && std::string(e.record().parameter) == "cuda.f32_variant is not a kernel family";
    }
    EXPECT(threw);
    // work split across the GPUs of a node
    using U2 = std::pair<uint64_t, uint64_t>;
    EXPECT((kernix::shard_window(16, 0, 3) == U2(0, 6)));
    EXPECT((kernix::shard_window(16, 2, 3) == U2(11, 5)));
    EXPECT((kernix::row_piece(8192, 8, 512) == U2(512, 2)));
    // no executors: refused before anything runs
    threw = false;
    try {
        kernix::gemm_sharded({}, {}, {}, {});
    } catch (const kernix::OpsError &e) {
        threw = e.status() == KX_E_PARAM;
    }
    EXPECT(threw);
}

static void gpu_checks() {
    kernix::CudaExecutor cuda(0);
    // ops_tests.rs:286-293: transpose view times F-order view
    auto x = cuda.upload<double>({1, 2, 3, 4}, {2, 2});
    auto yf = cuda.upload<double>({5, 7, 6, 8}, {2, 2}).transpose();   // F-order [[5,6],[7,8]]
    auto z = cuda.matmul(x.transpose(), yf);
    auto zv = cuda.download(z);
    EXPECT(zv.size() == 4 && zv[0] == 26 && zv[1] == 30 && zv[2] == 38 && zv[3] == 44);
    // batched_matmul_tests.rs:49-65: swapped then reversed batch view, ordered == exact
    std::vector<double> base(24);
    for (int i = 0; i < 24; ++i) base[i] = i / 16.0;
    auto t = cuda.upload<double>(base, {2, 3, 4}).swap_axes(1, 2).reverse_axis(2);
    auto bm = cuda.upload<double>(std::vector<double>(6, 0.75), {3, 2});
    auto p = cuda.matmul(t, bm);
    auto pv = cuda.download(p);
    EXPECT(pv.size() == 16);
    for (int bi = 0; bi < 2; ++bi)
        for (int i = 0; i < 4; ++i) {
            double s = 0;
            for (int k = 0; k < 3; ++k) s += base[bi * 12 + (2 - k) * 4 + i] * 0.75;   // dyadic: exact
            EXPECT(pv[(bi * 4 + i) * 2] == s && pv[(bi * 4 + i) * 2 + 1] == s);
        }
    // MatmulElement hooks on host buffers (small_matmul_tests.rs dyadic data, exact)
    kernix::Handle h(0);
    const size_t m = 17, k = 33, n = 9;
    std::vector<float> av(m * k), bv(k * n), ov(m * n + 2, NAN);
    for (size_t i = 0; i < av.size(); ++i) av[i] = ((i * 7 % 29) - 14.0f) / 8.0f;
    for (size_t i = 0; i < bv.size(); ++i) bv[i] = ((i * 11 % 37) - 18.0f) / 16.0f;
    EXPECT(kernix::MatmulElement<float>::try_dense_matmul(h, av.data(), av.size(), bv.data(), bv.size(),
                                                          ov.data() + 1, m * n, m, k, n));
    for (size_t i = 0; i < m; ++i)
        for (size_t j = 0; j < n; ++j) {
            double s = 0;
            for (size_t q = 0; q < k; ++q) s += (double)av[i * k + q] * bv[q * n + j];
            EXPECT((double)ov[1 + i * n + j] == s);
        }
    EXPECT(std::isnan(ov[0]) && std::isnan(ov[m * n + 1]));
    auto ma = kernix::MatrixInput<float>::create(av.data(), av.size(), {m, k}, {(std::ptrdiff_t)k, 1}, 0);
    auto mb = kernix::MatrixInput<float>::create(bv.data(), bv.size(), {k, n}, {(std::ptrdiff_t)n, 1}, 0);
    std::vector<float> o2(m * n);
    EXPECT(kernix::MatmulElement<float>::try_strided_matmul(h, ma, mb, o2.data(), o2.size()));
    for (size_t i = 0; i < m * n; ++i) EXPECT(o2[i] == ov[1 + i]);
    // ordered mode is available and reported
    cuda.with_ordered_matmul(true);
    EXPECT(cuda.ordered_matmul());
    cuda.with_ordered_matmul(false);
    // tensordot (ops_completeness_03.rs:224-237)
    auto tx = cuda.upload<double>({1, 2, 3, 4, 5, 6}, {2, 3});
    auto ty = cuda.upload<double>({1, 0, 0, 0, 1, 0, 0, 0, 1, 1, 1, 1}, {4, 3});
    auto tz = cuda.download(cuda.tensordot(tx, ty, {1}, {1}));
    EXPECT(tz == std::vector<double>({1, 2, 3, 6, 4, 5, 6, 15}));
    // softmax of [0, ln 3]: [1/4, 3/4] (math.rs:531-536)
    auto sm = cuda.download(cuda.softmax(cuda.upload<double>({0.0, std::log(3.0)}, {1, 2}), -1));
    EXPECT(std::fabs(sm[0] - 0.25) < 1e-15 && std::fabs(sm[1] - 0.75) < 1e-15);
    // matmul VJP with grad = ones: dA rows are B's row sums, dB columns A's column sums (exact)
    auto va = cuda.upload<double>({1, 2, 3, 4, 5, 6}, {2, 3});
    auto vb = cuda.upload<double>({0.5, -1, 2, 0.25, 1, 1}, {3, 2});
    auto g = cuda.matmul_backward(va, vb, cuda.upload<double>({1, 1, 1, 1}, {2, 2}));
    EXPECT(cuda.download(g.first) == std::vector<double>({-0.5, 2.25, 2, -0.5, 2.25, 2}));
    EXPECT(cuda.download(g.second) == std::vector<double>({5, 5, 7, 7, 9, 9}));
    // attention products against the host: out = softmax(q k^T / T) v
    const int sq = 5, sk = 7, d = 128;
    std::vector<float> q(sq * d), kk(sk * d), v(sk * d);
    for (int i = 0; i < sq * d; ++i) q[i] = (float)((i * 37 % 101) - 50) / 64.0f;
    for (int i = 0; i < sk * d; ++i) kk[i] = (float)((i * 53 % 97) - 48) / 64.0f;
    for (int i = 0; i < sk * d; ++i) v[i] = (float)((i * 29 % 89) - 44) / 32.0f;
    const float temp = 11.3137085f;
    auto dq = cuda.upload<float>(q, {1, (uint64_t)sq, (uint64_t)d});
    auto dkt = cuda.upload<float>(kk, {1, (uint64_t)sk, (uint64_t)d}).swap_axes(1, 2);
    auto dv = cuda.upload<float>(v, {1, (uint64_t)sk, (uint64_t)d});
    auto att = cuda.download(cuda.attention(dq, dkt, dv, temp));
    for (int i = 0; i < sq; ++i) {
        std::vector<double> s(sk), pr(sk);
        double mx = -1e300, sum = 0;
        for (int j = 0; j < sk; ++j) {
            for (int c = 0; c < d; ++c) s[j] += (double)q[i * d + c] * kk[j * d + c];
            mx = std::max(mx, s[j]);
        }
        for (int j = 0; j < sk; ++j) sum += (pr[j] = std::exp((s[j] - mx) / temp));
        for (int c = 0; c < d; ++c) {
            double o = 0, ab = 0;
            for (int j = 0; j < sk; ++j) {
                o += pr[j] / sum * v[j * d + c];
                ab += pr[j] / sum * std::fabs(v[j * d + c]);
            }
            EXPECT(std::fabs(att[i * d + c] - o) <= 1e-4 * ab + 1e-12);
        }
    }
    // a context from the [cuda] table: ordered products (bit for bit the ordered sums)
    kernix::CudaConfig cfg;
    cfg.c.ordered_matmul = 1;
    kernix::CudaExecutor ordered(cfg);
    EXPECT(ordered.ordered_matmul());
    kernix::Handle hc(cfg);
    EXPECT(hc.config().c.ordered_matmul == 1 && hc.config().c.device == 0);
    auto oa = ordered.upload<float>({0.1f, 0.2f, 0.3f}, {1, 3});
    auto ob = ordered.upload<float>({0.7f, 0.11f, 0.13f}, {3, 1});
    auto ov1 = ordered.download(ordered.matmul(oa, ob));
    float acc = 0.0f;
    const float ta[3] = {0.1f, 0.2f, 0.3f}, tb[3] = {0.7f, 0.11f, 0.13f};
    for (int i = 0; i < 3; ++i) {
        volatile float prod = ta[i] * tb[i];        // separately rounded, as matmul_reference
        acc = acc + prod;
    }
    EXPECT(ov1.size() == 1 && ov1[0] == acc);
    // one process over two executors (both on device 0 here): windows of 3
    // and 2 rows, every output gathered to the whole product
    {
        const uint64_t m = 5, k = 7, n = 6;
        std::vector<float> av(m * k), bv(k * n);
        for (size_t i = 0; i < av.size(); ++i) av[i] = (float)((int)(i % 9) - 4) / 4.0f;
        for (size_t i = 0; i < bv.size(); ++i) bv[i] = (float)((int)(i % 5) - 2) / 2.0f;
        kernix::CudaExecutor e0(0), e1(0);
        std::vector<const kernix::CudaExecutor *> ex = {&e0, &e1};
        std::vector<kernix::DeviceTensor<float>> aw, br, outs;
        for (uint32_t r = 0; r < 2; ++r) {
            auto w = kernix::shard_window(m, r, 2);
            const kernix::CudaExecutor &x = *ex[r];
            aw.push_back(x.upload<float>(std::vector<float>(av.begin() + w.first * k,
                                                            av.begin() + (w.first + w.second) * k),
                                         {w.second, k}));
            br.push_back(x.upload<float>(bv, {k, n}));
            outs.push_back(x.upload<float>(std::vector<float>(m * n, -1.0f), {m, n}));
        }
        kernix::gemm_sharded(ex, aw, br, outs, true);
        e0.synchronize();
        e1.synchronize();
        auto o0 = e0.download(outs[0]), o1 = e1.download(outs[1]);
        bool exact = o0 == o1;
        for (uint64_t i = 0; i < m; ++i)
            for (uint64_t j = 0; j < n; ++j) {
                double s = 0;       // dyadic data: every product and sum is exact in f32
                for (uint64_t q = 0; q < k; ++q) s += (double)av[i * k + q] * bv[q * n + j];
                exact = exact && (double)o0[i * n + j] == s;
            }
        EXPECT(exact);
    }
}

int main(int argc, char **argv) {
    bool gpu = argc > 1 && std::string(argv[1]) == "--gpu";
    host_checks();
    if (gpu) gpu_checks();
    if (failures) {
        std::fprintf(stderr, "%d failure(s)\n", failures);
        return 1;
    }
    std::printf("mirror_test ok (%s)\n", gpu ? "host+gpu" : "host");
    return 0;
}
