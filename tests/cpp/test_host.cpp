// test_host.cpp — the C++ host mirror (go-whistle_b200/host/whistle.hpp)
// tested the way the reference tests internal/cq and internal/needle, the
// GPU results checked against the CPU oracle (oracle/oracle.h, test
// infrastructure) bit for bit.
//
//   test_host --cpu   tests that need no GPU (validation, panics, helpers)
//   test_host --gpu   parity tests on the GPU
// Exit status 0 when every test passes.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <random>
#include <string>
#include <vector>

#include "oracle.h"
#include "whistle.hpp"

using namespace whistle;

namespace {

int g_failures = 0;
std::string g_test;

#define EXPECT(cond)                                                                          \
    do {                                                                                      \
        if (!(cond)) {                                                                        \
            std::fprintf(stderr, "%s: %s:%d: expected %s\n", g_test.c_str(), __FILE__, __LINE__, #cond); \
            g_failures++;                                                                     \
        }                                                                                     \
    } while (0)

template <class E, class F>
bool throws_with(F f, const std::string &text) {
    try {
        f();
    } catch (const E &e) {
        if (std::string(e.what()).find(text) == std::string::npos) {
            std::fprintf(stderr, "%s: message \"%s\" lacks \"%s\"\n", g_test.c_str(), e.what(), text.c_str());
            return false;
        }
        return true;
    } catch (const std::exception &e) {
        std::fprintf(stderr, "%s: wrong exception: %s\n", g_test.c_str(), e.what());
        return false;
    }
    std::fprintf(stderr, "%s: no exception\n", g_test.c_str());
    return false;
}

bool same_bits(const float *a, const float *b, size_t n) { return std::memcmp(a, b, n * sizeof(float)) == 0; }

// A random CQ tensor as the reference's tests draw one (cq_test.go:30-38):
// uniform codes, a sorted codebook, FP16 norms 2^-4 .. 2^4.
cq::Packed random_packed(std::mt19937_64 &rng, int out, int in, int group, int bits) {
    cq::Packed p;
    p.Out = out;
    p.In = in;
    p.Group = group;
    p.Bits = bits;
    p.Width = bits;
    std::normal_distribution<float> nd(0.0f, 0.02f);
    for (int c = 0; c < (1 << bits); c++) p.Codebook.push_back(nd(rng));
    std::sort(p.Codebook.begin(), p.Codebook.end());
    p.Index.resize((size_t)out * p.RowBytes());
    for (auto &b : p.Index) b = (uint8_t)(rng() & 0xff);
    p.Norms.resize((size_t)2 * out * p.Groups());
    for (size_t i = 0; i < p.Norms.size(); i += 2) {
        const uint16_t h = (uint16_t)(((11 + rng() % 9) << 10) | (rng() & 1023));  // exponent 11..19
        p.Norms[i] = (uint8_t)(h & 0xff);
        p.Norms[i + 1] = (uint8_t)(h >> 8);
    }
    return p;
}

wo_packed as_oracle(const cq::Packed &p) {
    return wo_packed{p.Out, p.In, p.Group, p.Bits, p.Index.data(), reinterpret_cast<const uint16_t *>(p.Norms.data()),
                     p.Codebook.data()};
}

std::vector<float> normal(std::mt19937_64 &rng, size_t n) {
    std::normal_distribution<float> nd(0.0f, 1.0f);
    std::vector<float> v(n);
    for (auto &x : v) x = nd(rng);
    return v;
}

// ---------------------------------------------------------------- CPU ----

// internal/cq/cq_test.go:561 TestNewErrors
void TestNewErrors() {
    std::mt19937_64 rng(7);
    const cq::Packed good = random_packed(rng, 2, 128, 128, 2);
    struct Case {
        const char *name;
        std::function<void(cq::Packed &)> edit;
        const char *want;
    } cases[] = {
        {"3 bits", [](cq::Packed &p) { p.Bits = p.Width = 3; }, "not supported"},
        {"ternary", [](cq::Packed &p) { p.Bits = 5; }, "not supported"},
        {"group 24", [](cq::Packed &p) { p.Group = 24; }, "power of two"},
        {"codebook", [](cq::Packed &p) { p.Codebook.resize(3); }, "codebook"},
        {"index", [](cq::Packed &p) { p.Index.pop_back(); }, "index"},
        {"norms", [](cq::Packed &p) { p.Norms.resize(p.Norms.size() - 2); }, "norm"},
    };
    for (auto &c : cases) {
        cq::Packed p = good;
        c.edit(p);
        EXPECT(throws_with<Error>([&] { cq::New(p); }, "cq: "));
        EXPECT(throws_with<Error>([&] { cq::New(p); }, c.want));
    }
}

// internal/cact/packed.go:32-40 Groups, RowBytes, Norm
void TestPackedHelpers() {
    cq::Packed p;
    p.Out = 1;
    p.In = 40;
    p.Group = 32;
    p.Bits = p.Width = 4;
    EXPECT(p.Groups() == 2);
    EXPECT(p.RowBytes() == 32);
    p.Norms = {0x00, 0x3c, 0x00, 0xc0};  // 1.0, -2.0
    EXPECT(p.Norm(0, 0) == 1.0f);
    EXPECT(p.Norm(0, 1) == -2.0f);
    for (uint32_t h = 0; h < 65536; h += 7) {  // internal/cact/half_test.go against the oracle's widening
        cq::Packed q = p;
        q.Norms = {(uint8_t)(h & 0xff), (uint8_t)(h >> 8), 0, 0};
        const float a = q.Norm(0, 0), b = wo_f16_to_f32((uint16_t)h);
        EXPECT(std::isnan(a) ? std::isnan(b) : std::memcmp(&a, &b, 4) == 0);
    }
}

// internal/needle/int8.go:107, 126: NewInt8Rows and Append reject bad shapes
void TestInt8RowsPanics() {
    EXPECT(throws_with<Panic>([] { needle::NewInt8Rows(10, 3); }, "needle: int8 rows of 10 in chunks of 3"));
    EXPECT(throws_with<Panic>([] { needle::NewInt8Rows(8, 0); }, "needle: "));
    needle::Int8Rows r = needle::NewInt8Rows(8, 4);
    std::vector<float> x(12, 1.0f);
    EXPECT(throws_with<Panic>([&] { r.Append(x.data(), x.size()); }, "needle: 12 values are not rows of 8"));
    EXPECT(r.Append(x.data(), 0).Len() == 0);
}

// ---------------------------------------------------------------- GPU ----

// internal/cq/kernel.go:101-107: shape misuse panics with gemm's text
void TestGEMMPanics() {
    std::mt19937_64 rng(3);
    cq::Matrix m = cq::New(random_packed(rng, 6, 64, 32, 4));
    std::vector<float> x(64 * 2), y(6 * 2);
    EXPECT(throws_with<Panic>([&] { m.GEMM(y.data(), 11, x.data(), 128, 2); }, "cq: GEMM(len 11, len 128, 2 rows) on [6, 64]"));
    EXPECT(throws_with<Panic>([&] { m.GEMM(y.data(), 12, x.data(), 127, 2); }, "cq: GEMM("));
    EXPECT(throws_with<Panic>([&] { m.GEMV(y.data(), 5, x.data(), 64); }, "cq: GEMM("));
    EXPECT(throws_with<Panic>([&] { m.Rows(4, 9); }, "cq: Rows(4, 9) of 6 rows"));
    EXPECT(throws_with<Panic>([&] { m.Row(y.data(), 64, 6); }, "cq: Row("));
    m.GEMM(y.data(), 0, x.data(), 0, 0);  // rows = 0 is a no-op (kernel.go:110)
}

// internal/cq/cq_test.go:196 TestKernels (lut and Exact), bit for bit
// against the oracle's restatement, on the reference's test shapes.
void TestKernels() {
    struct Shape {
        int out, in, group;
    } shapes[] = {{1, 8, 8}, {3, 16, 8}, {5, 40, 32}, {7, 200, 128}, {33, 256, 128}, {384, 512, 128}, {2048, 512, 32},
                  {512, 2048, 32}};
    std::mt19937_64 rng(11);
    for (int bits : {2, 4}) {
        for (auto s : shapes) {
            const cq::Packed p = random_packed(rng, s.out, s.in, s.group, bits);
            cq::Matrix m = cq::New(p);
            const wo_packed o = as_oracle(p);
            for (int rows : {1, 3}) {
                const std::vector<float> x = normal(rng, (size_t)rows * s.in);
                std::vector<float> got((size_t)rows * s.out), want(got.size());
                m.GEMM(got.data(), got.size(), x.data(), x.size(), rows);
                EXPECT(wo_cq_gemm_lut(&o, x.data(), rows, want.data()) == 0);
                EXPECT(same_bits(got.data(), want.data(), got.size()));
                cq::Matrix e = m.Exact();
                e.GEMM(got.data(), got.size(), x.data(), x.size(), rows);
                wo_cq_gemm_exact(&o, x.data(), rows, want.data());
                EXPECT(same_bits(got.data(), want.data(), got.size()));
            }
        }
    }
}

// internal/cq/parallel_test.go:101 TestGEMMsMatchesGEMM, and views
// (matrix.go:133 Rows) against their parent's rows
void TestGEMMsAndRows() {
    std::mt19937_64 rng(21);
    std::vector<cq::Packed> ps;
    for (int o : {384, 96, 128, 512}) ps.push_back(random_packed(rng, o, 512, 128, 2));
    for (auto &p : ps) p.Codebook = ps[0].Codebook;
    std::vector<cq::Matrix> ms;
    for (auto &p : ps) ms.push_back(cq::New(p));
    const int rows = 2;
    const std::vector<float> x = normal(rng, (size_t)rows * 512);
    std::vector<std::vector<float>> ys(ms.size());
    std::vector<cq::Slice> dsts;
    for (size_t k = 0; k < ms.size(); k++) {
        ys[k].assign((size_t)rows * ms[k].Out(), NAN);
        dsts.push_back({ys[k].data(), ys[k].size()});
    }
    cq::GEMMs(ms, dsts, x.data(), x.size(), rows);
    for (size_t k = 0; k < ms.size(); k++) {
        std::vector<float> one(ys[k].size());
        ms[k].GEMM(one.data(), one.size(), x.data(), x.size(), rows);
        EXPECT(same_bits(one.data(), ys[k].data(), one.size()));
    }
    cq::Matrix v = ms[3].Rows(100, 300);
    EXPECT(v.Out() == 200 && v.In() == 512 && v.Bits() == 2);
    std::vector<float> yv((size_t)rows * 200);
    v.GEMM(yv.data(), yv.size(), x.data(), x.size(), rows);
    for (int r = 0; r < rows; r++) EXPECT(same_bits(yv.data() + r * 200, ys[3].data() + r * 512 + 100, 200));
}

// internal/cq/cq_test.go TestRow: Row equals the oracle's dequantisation
void TestRow() {
    std::mt19937_64 rng(5);
    for (int bits : {2, 4}) {
        const cq::Packed p = random_packed(rng, 9, 200, 64, bits);
        cq::Matrix m = cq::New(p);
        const wo_packed o = as_oracle(p);
        std::vector<float> got(200), want(200);
        for (int r = 0; r < 9; r++) {
            m.Row(got.data(), got.size(), r);
            wo_cq_row(&o, r, want.data());
            EXPECT(same_bits(got.data(), want.data(), 200));
        }
    }
}

// internal/needle/int8_test.go:16 TestQuantizeRow's literal cases
void TestQuantizeRow() {
    int8_t q[6];
    const float a[6] = {127, 2.5f, -2.5f, 3.5f, -0.5f, 1.4999f};
    EXPECT(needle::QuantizeRow(q, 6, a, 6) == 1.0f);
    const int8_t wa[6] = {127, 2, -2, 4, 0, 1};
    EXPECT(std::memcmp(q, wa, 6) == 0);
    const float b[3] = {-6.35f, 0.05f, 3};
    EXPECT(needle::QuantizeRow(q, 6, b, 3) == 6.35f / 127.0f);
    const int8_t wb[3] = {-127, 1, 60};
    EXPECT(std::memcmp(q, wb, 3) == 0);
    const float z[4] = {0, 0, 0, 0};
    EXPECT(needle::QuantizeRow(q, 6, z, 4) == 1.0f);
    EXPECT(throws_with<Panic>([&] { needle::QuantizeRow(q, 2, z, 4); }, "needle: QuantizeRow"));
}

// internal/needle/int8_test.go:212 TestAttendInt8MatchesFloat: the GPU
// equals the oracle bit for bit (quantQ on and off, causal and full), and
// each row's weights sum to 1 within 1e-5.
void TestAttendInt8() {
    std::mt19937_64 rng(9);
    const int heads = 8, kvh = 2, qk = 48, vd = 64, n = 37, t = 3;
    const std::vector<float> q = normal(rng, (size_t)t * heads * qk);
    const std::vector<float> kf = normal(rng, (size_t)n * kvh * qk), vf = normal(rng, (size_t)n * kvh * vd);
    const needle::Int8Rows k = needle::QuantizeRows(kf.data(), kf.size(), kvh * qk, qk);
    const needle::Int8Rows v = needle::QuantizeRows(vf.data(), vf.size(), kvh * vd, vd);
    EXPECT(k.Len() == n && v.Len() == n && k.Bytes() == (size_t)n * kvh * qk + 4 * (size_t)n * kvh);
    std::vector<int8_t> q8(kf.size());
    std::vector<float> s8(k.S.size());
    wo_quantize_rows(kf.data(), n, kvh * qk, qk, q8.data(), s8.data());
    EXPECT(std::memcmp(q8.data(), k.Q.data(), q8.size()) == 0 && same_bits(s8.data(), k.S.data(), s8.size()));
    const float scale = std::sqrt((float)qk);
    for (bool causal : {false, true}) {
        for (bool quantQ : {true, false}) {
            auto keys = [&](int i) { return causal ? n - t + i + 1 : n; };
            std::vector<float> probs((size_t)t * heads * n, 0.0f), wprobs(probs.size(), 0.0f);
            const std::vector<float> got =
                needle::AttendInt8(q.data(), q.size(), t, heads, k, v, keys, scale, quantQ, probs.data(), probs.size());
            std::vector<int32_t> sp;
            for (int i = 0; i < t; i++) sp.insert(sp.end(), {0, 0, 0, keys(i)});
            std::vector<float> want((size_t)t * heads * vd, 0.0f);
            wo_attend_int8_spans(q.data(), t, heads, k.Q.data(), k.S.data(), v.Q.data(), v.S.data(), n, kvh, qk, vd,
                                 sp.data(), scale, quantQ ? 1 : 0, wprobs.data(), want.data());
            EXPECT(same_bits(got.data(), want.data(), got.size()));
            EXPECT(same_bits(probs.data(), wprobs.data(), probs.size()));
            for (int i = 0; i < t; i++)
                for (int h = 0; h < heads; h++) {
                    double sum = 0;
                    for (int j = 0; j < keys(i); j++) sum += probs[((size_t)i * heads + h) * n + j];
                    EXPECT(std::fabs(sum - 1.0) <= 1e-5);
                }
        }
    }
}

void run(const char *name, void (*f)()) {
    g_test = name;
    const int before = g_failures;
    try {
        f();
    } catch (const std::exception &e) {
        std::fprintf(stderr, "%s: unexpected exception: %s\n", name, e.what());
        g_failures++;
    }
    std::printf("%s %s\n", g_failures == before ? "PASS" : "FAIL", name);
}

}  // namespace

int main(int argc, char **argv) {
    const bool cpu = argc > 1 && std::strcmp(argv[1], "--cpu") == 0;
    const bool gpu = argc > 1 && std::strcmp(argv[1], "--gpu") == 0;
    if (!cpu && !gpu) {
        std::fprintf(stderr, "usage: test_host --cpu | --gpu\n");
        return 2;
    }
    if (cpu) {
        run("TestNewErrors", TestNewErrors);
        run("TestPackedHelpers", TestPackedHelpers);
        run("TestInt8RowsPanics", TestInt8RowsPanics);
    } else {
        run("TestGEMMPanics", TestGEMMPanics);
        run("TestKernels", TestKernels);
        run("TestGEMMsAndRows", TestGEMMsAndRows);
        run("TestRow", TestRow);
        run("TestQuantizeRow", TestQuantizeRow);
        run("TestAttendInt8", TestAttendInt8);
    }
    return g_failures == 0 ? 0 : 1;
}
