// whistle.hpp — the host side of go-whistle's quantized hot path in C++,
// over the C ABI of libwhistle_b200.so (include/whistle_b200.h).
//
// It mirrors the reference's Go API for the path name for name, with the
// same argument meaning and error behaviour:
//   internal/cq     Packed, New, NewGather, Matrix (Out, In, Bits, Bytes,
//                   Prepare, Rows, Exact, Row, GEMV, GEMM), GEMMs
//   internal/needle QuantizeRow, NewInt8Rows, QuantizeRows, Int8Rows
//                   (Append, Len, Floats, Bytes), Span, AttendInt8,
//                   AttendInt8Spans
// Where Go returns an error this throws whistle::Error with the reference's
// text ("cq: ..."); where Go panics on misuse it throws whistle::Panic with
// the panic text; CUDA failures throw whistle::CudaError. Slices are
// (pointer, length) pairs in host memory, as the Go shim passes them; every
// product runs on the GPU, and a call returns when its result is in the
// caller's memory. Nothing here computes.
#pragma once

#include <array>
#include <cstddef>
#include <cstdint>
#include <functional>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "whistle_b200.h"

namespace whistle {

// A failed call; status() is the wc_status code.
class Failure : public std::runtime_error {
   public:
    Failure(int status, const std::string &msg) : std::runtime_error(msg), status_(status) {}
    int status() const { return status_; }

   private:
    int status_;
};
struct Error : Failure {  // what the reference returns as an error
    using Failure::Failure;
};
struct Panic : Failure {  // what the reference panics on
    using Failure::Failure;
};
struct CudaError : Failure {  // a CUDA failure, or a handle used on the wrong device
    using Failure::Failure;
};

// Throws the exception a non-zero status stands for, with the library's
// message.
void check(wc_status st);

namespace cq {

// cact.Packed (internal/cact/packed.go:18-40): a CQ tensor as stored.
struct Packed {
    int Out = 0, In = 0, Group = 0, Bits = 0, Width = 0;
    std::vector<float> Codebook;
    std::vector<uint8_t> Index;  // Out rows of RowBytes() LSB-first indices
    std::vector<uint8_t> Norms;  // Out·Groups() FP16 values, little-endian
    int Groups() const { return (In + Group - 1) / Group; }          // packed.go:32
    int RowBytes() const { return Groups() * Group * Width / 8; }     // packed.go:35
    float Norm(int r, int g) const;                                   // packed.go:38
};

// internal/cq/matrix.go:25 Matrix: [Out, In], resident on the GPU current
// when it was made. Copies share the device storage; safe for concurrent
// use.
class Matrix {
   public:
    Matrix() = default;
    int Out() const;   // matrix.go:99
    int In() const;    // matrix.go:102
    int Bits() const;  // matrix.go:105
    size_t Bytes() const;
    void Prepare() const {}  // matrix.go:111: New made the device copy
    Matrix Rows(int lo, int hi) const;  // matrix.go:133
    Matrix Exact() const;               // matrix.go:152
    // matrix.go:161 Row: dst (In values) gets row r dequantised exactly.
    void Row(float *dst, size_t dst_len, int r) const;
    // kernel.go:78 GEMV: dst (Out values) = W·x (In values).
    void GEMV(float *dst, size_t dst_len, const float *x, size_t x_len) const;
    // kernel.go:85 GEMM: dst[rows·Out] = x[rows·In] · Wᵀ; rows = 0 is a no-op.
    void GEMM(float *dst, size_t dst_len, const float *x, size_t x_len, int rows) const;
    const wc_cq *handle() const { return h_.get(); }

   private:
    friend Matrix New(const Packed &p);
    explicit Matrix(wc_cq *h);
    std::shared_ptr<wc_cq> h_;
};

Matrix New(const Packed &p);        // matrix.go:46
inline Matrix NewGather(const Packed &p) { return New(p); }  // matrix.go:60: no separate CPU layout here

// A destination slice of GEMMs.
struct Slice {
    float *p;
    size_t n;
};
// kernel.go:134 GEMMs: dsts[k] = x · ms[k]ᵀ, the tables of matrices that
// share them built once.
void GEMMs(const std::vector<Matrix> &ms, const std::vector<Slice> &dsts, const float *x, size_t x_len, int rows);

}  // namespace cq

namespace needle {

// int8.go:36 QuantizeRow: q (at least n codes) gets x's codes; returns the scale.
float QuantizeRow(int8_t *q, size_t q_len, const float *x, size_t n);

// int8.go:99 Int8Rows: rows of Cols int8 codes, one float32 scale per chunk
// of Width codes. Append returns a new value, as Go's does.
struct Int8Rows {
    int Cols = 0, Width = 0;
    std::vector<int8_t> Q;
    std::vector<float> S;
    int Len() const { return Cols == 0 ? 0 : (int)(Q.size() / (size_t)Cols); }  // int8.go:144
    Int8Rows Append(const float *x, size_t n) const;                             // int8.go:125
    std::vector<float> Floats() const;                                           // int8.go:163
    size_t Bytes() const { return Q.size() + 4 * S.size(); }                     // int8.go:174
};
Int8Rows NewInt8Rows(int cols, int width);                            // int8.go:107
Int8Rows QuantizeRows(const float *x, size_t n, int cols, int width);  // int8.go:116

struct Span {  // key rows [Lo, Hi)
    int Lo = 0, Hi = 0;
    int Len() const { return Hi - Lo; }
};

// int8.go:208 AttendInt8Spans: t query rows of heads·k.Width values; row i
// sees the keys of the two spans spans(i). probs (or nullptr) receives the
// weights at (i·heads + h)·k.Len() + j, at the spans' keys only.
std::vector<float> AttendInt8Spans(const float *q, size_t q_len, int t, int heads, const Int8Rows &k,
                                   const Int8Rows &v, const std::function<std::array<Span, 2>(int)> &spans,
                                   float scale, bool quantQ, float *probs, size_t probs_len);

// int8.go:194 AttendInt8: row i sees the first keys(i) rows.
std::vector<float> AttendInt8(const float *q, size_t q_len, int t, int heads, const Int8Rows &k, const Int8Rows &v,
                              const std::function<int(int)> &keys, float scale, bool quantQ, float *probs,
                              size_t probs_len);

}  // namespace needle
}  // namespace whistle
