// whistle.cpp — the C++ host mirror of internal/cq and internal/needle over
// the C ABI (whistle.hpp says what each routine stands in for).
#include "whistle.hpp"

#include <cstring>

namespace whistle {

namespace {
std::string last_error() {
    char buf[1024];
    wc_last_error(buf, sizeof buf);
    return buf;
}
}  // namespace

void check(wc_status st) {
    switch (st) {
        case WC_OK:
            return;
        case WC_ERR_INVALID:
            throw Panic(st, last_error());
        case WC_ERR_UNSUPPORTED:
            throw Error(st, last_error());
        default:
            throw CudaError(st, last_error());
    }
}

namespace cq {

float Packed::Norm(int r, int g) const {
    const size_t o = 2 * ((size_t)r * Groups() + g);
    const uint16_t h = (uint16_t)(Norms.at(o) | (Norms.at(o + 1) << 8));
    // IEEE half to float (internal/cact/half.go): exact.
    const uint32_t sign = (uint32_t)(h >> 15) << 31, exp = (h >> 10) & 31, man = h & 1023;
    uint32_t bits;
    if (exp == 0 && man == 0) {
        bits = sign;
    } else if (exp == 0) {  // subnormal: normalise
        int e = -1;
        uint32_t m = man;
        do {
            e++;
            m <<= 1;
        } while (!(m & 1024));
        bits = sign | (uint32_t)(127 - 15 - e) << 23 | (m & 1023) << 13;
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | man << 13;
    } else {
        bits = sign | (exp + 127 - 15) << 23 | man << 13;
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

Matrix::Matrix(wc_cq *h) : h_(h, [](wc_cq *p) { wc_cq_destroy(p); }) {}

int Matrix::Out() const { return wc_cq_out(h_.get()); }
int Matrix::In() const { return wc_cq_in(h_.get()); }
int Matrix::Bits() const { return wc_cq_bits(h_.get()); }
size_t Matrix::Bytes() const { return wc_cq_bytes(h_.get()); }

Matrix Matrix::Rows(int lo, int hi) const {
    wc_cq *v = nullptr;
    check(wc_cq_rows(h_.get(), lo, hi, &v));
    return Matrix(v);
}

Matrix Matrix::Exact() const {
    wc_cq *v = nullptr;
    check(wc_cq_exact(h_.get(), &v));
    return Matrix(v);
}

void Matrix::Row(float *dst, size_t dst_len, int r) const { check(wc_cq_row_host(h_.get(), r, dst, dst_len)); }

void Matrix::GEMV(float *dst, size_t dst_len, const float *x, size_t x_len) const { GEMM(dst, dst_len, x, x_len, 1); }

void Matrix::GEMM(float *dst, size_t dst_len, const float *x, size_t x_len, int rows) const {
    check(wc_cq_gemm_host(h_.get(), x, x_len, dst, dst_len, rows));
}

Matrix New(const Packed &p) {
    wc_cq *h = nullptr;
    check(wc_cq_create(p.Index.data(), p.Index.size(), p.Norms.data(), p.Norms.size(), p.Codebook.data(),
                       p.Codebook.size(), p.Out, p.In, p.Group, p.Bits, p.Width, &h));
    return Matrix(h);
}

void GEMMs(const std::vector<Matrix> &ms, const std::vector<Slice> &dsts, const float *x, size_t x_len, int rows) {
    if (ms.size() != dsts.size())
        throw Panic(WC_ERR_INVALID, "cq: GEMMs of " + std::to_string(ms.size()) + " matrices into " +
                                        std::to_string(dsts.size()) + " outputs");
    std::vector<const wc_cq *> hs(ms.size());
    std::vector<float *> ys(ms.size());
    std::vector<size_t> lens(ms.size());
    for (size_t k = 0; k < ms.size(); k++) {
        hs[k] = ms[k].handle();
        ys[k] = dsts[k].p;
        lens[k] = dsts[k].n;
    }
    check(wc_cq_gemms_host(hs.data(), (int)hs.size(), x, x_len, ys.data(), lens.data(), rows));
}

}  // namespace cq

namespace needle {

float QuantizeRow(int8_t *q, size_t q_len, const float *x, size_t n) {
    if (q_len < n)
        throw Panic(WC_ERR_INVALID,
                    "needle: QuantizeRow into " + std::to_string(q_len) + " codes of " + std::to_string(n) + " values");
    if (n == 0) return 1.0f;  // int8.go:40: the scale of an empty or zero row is 1
    float s = 0.0f;
    check(wc_quantize_rows_host(x, n, (int)n, (int)n, q, &s));
    return s;
}

Int8Rows NewInt8Rows(int cols, int width) {
    if (width <= 0 || cols % width != 0)
        throw Panic(WC_ERR_INVALID,
                    "needle: int8 rows of " + std::to_string(cols) + " in chunks of " + std::to_string(width));
    Int8Rows r;
    r.Cols = cols;
    r.Width = width;
    return r;
}

Int8Rows Int8Rows::Append(const float *x, size_t n) const {
    if (Cols == 0 || n % (size_t)Cols != 0)
        throw Panic(WC_ERR_INVALID,
                    "needle: " + std::to_string(n) + " values are not rows of " + std::to_string(Cols));
    Int8Rows r = *this;
    if (n == 0) return r;
    const size_t q0 = r.Q.size(), s0 = r.S.size();
    r.Q.resize(q0 + n);
    r.S.resize(s0 + n / Width);
    check(wc_quantize_rows_host(x, n, Cols, Width, r.Q.data() + q0, r.S.data() + s0));
    return r;
}

std::vector<float> Int8Rows::Floats() const {
    std::vector<float> f(Q.size());
    for (size_t i = 0; i < Q.size(); i++) f[i] = (float)Q[i] * S[i / Width];
    return f;
}

Int8Rows QuantizeRows(const float *x, size_t n, int cols, int width) { return NewInt8Rows(cols, width).Append(x, n); }

std::vector<float> AttendInt8Spans(const float *q, size_t q_len, int t, int heads, const Int8Rows &k,
                                   const Int8Rows &v, const std::function<std::array<Span, 2>(int)> &spans,
                                   float scale, bool quantQ, float *probs, size_t probs_len) {
    if (k.Width <= 0 || v.Width <= 0 || k.Cols % k.Width != 0)
        throw Panic(WC_ERR_INVALID, "needle: AttendInt8 on empty int8 rows");
    const int qk = k.Width, vd = v.Width, kv_heads = k.Cols / qk;
    std::vector<int32_t> sp((size_t)(t > 0 ? t : 0) * 4);
    for (int i = 0; i < t; i++) {
        const std::array<Span, 2> s = spans(i);
        sp[4 * i] = s[0].Lo;
        sp[4 * i + 1] = s[0].Hi;
        sp[4 * i + 2] = s[1].Lo;
        sp[4 * i + 3] = s[1].Hi;
    }
    std::vector<float> out((size_t)(t > 0 ? t : 0) * heads * vd);
    check(wc_attend_int8_host(q, q_len, t, heads, k.Q.data(), k.Q.size(), k.S.data(), k.S.size(), v.Q.data(),
                              v.Q.size(), v.S.data(), v.S.size(), kv_heads, qk, vd, sp.data(), scale,
                              quantQ ? WC_ATTEND_QUANT_Q : 0, probs, probs_len, out.data(), out.size()));
    return out;
}

std::vector<float> AttendInt8(const float *q, size_t q_len, int t, int heads, const Int8Rows &k, const Int8Rows &v,
                              const std::function<int(int)> &keys, float scale, bool quantQ, float *probs,
                              size_t probs_len) {
    return AttendInt8Spans(
        q, q_len, t, heads, k, v, [&](int i) { return std::array<Span, 2>{Span{}, Span{0, keys(i)}}; }, scale, quantQ,
        probs, probs_len);
}

}  // namespace needle
}  // namespace whistle
