// bc_ops.hpp -- C++ host API mirroring barraCuda's FHE op interface
// (crates/barracuda/src/ops/fhe_*.rs) on top of the CUDA path.
//
// Same constructors, argument meaning, validation order and error text as
// the Rust ops; `execute` runs on the device's stream and returns once the
// result is complete, like the reference's submit + poll.
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <utility>
#include <vector>

#include "barracuda_fhe.h"

namespace barracuda {

// Mirrors BarracudaError (crates/barracuda/src/error.rs); `kind` is the C
// ABI status code of the variant.
struct Error {
    int kind = BC_OK;
    std::string message;
    // Rust Display text, e.g. "Device error: Modulus must be non-zero".
    std::string to_string() const;
};

template <class T>
class Result {
public:
    static Result ok(T v) { return Result(std::move(v)); }
    static Result err(Error e) { return Result(std::move(e)); }
    bool is_ok() const { return err_.kind == BC_OK; }
    bool is_err() const { return !is_ok(); }
    T &value() { return *val_; }
    T take() { return std::move(*val_); }
    const Error &error() const { return err_; }

private:
    explicit Result(T v) : val_(std::make_shared<T>(std::move(v))) {}
    explicit Result(Error e) : err_(std::move(e)) {}
    std::shared_ptr<T> val_;
    Error err_;
};

// One CUDA device (WgpuDevice's role for this path).
class Device {
public:
    static Result<std::shared_ptr<Device>> open(int ordinal);
    ~Device();
    bc_ctx *ctx() const { return ctx_; }

private:
    explicit Device(bc_ctx *c) : ctx_(c) {}
    bc_ctx *ctx_;
};

// Device buffer of u32 words (Tensor's role for this path): a polynomial of
// degree N is 2N words, [lo32, hi32] per coefficient.
class Tensor {
public:
    static Result<Tensor> from_u32(const std::vector<uint32_t> &data, std::shared_ptr<Device> dev);
    static Result<Tensor> empty_u64(size_t n_u64, std::shared_ptr<Device> dev);
    size_t len() const { return len_u32_; }
    const std::shared_ptr<Device> &device() const { return dev_; }
    const uint64_t *data() const { return static_cast<const uint64_t *>(buf_.get()); }
    uint64_t *mutable_data() const { return static_cast<uint64_t *>(buf_.get()); }
    Result<std::vector<uint32_t>> to_vec_u32() const;

private:
    std::shared_ptr<Device> dev_;
    std::shared_ptr<void> buf_;
    size_t len_u32_ = 0;
};

// ops/fhe_poly_add.rs:185 create_fhe_poly_tensor.
Result<Tensor> create_fhe_poly_tensor(const std::vector<uint64_t> &poly, std::shared_ptr<Device> dev);
// ops/fhe_ntt/mod.rs:210 compute_primitive_root.
uint64_t compute_primitive_root(uint32_t degree, uint64_t modulus);
// ops/fhe_intt/mod.rs:202 compute_inverse_root.
uint64_t compute_inverse_root(uint32_t degree, uint64_t modulus, uint64_t root);

// ops/fhe_ntt/mod.rs:71-171, compute.rs:29-143.
class FheNtt {
public:
    static Result<FheNtt> create(Tensor input, uint32_t degree, uint64_t modulus, uint64_t root_of_unity);
    Result<Tensor> execute() &&;

private:
    Tensor input_;
    uint32_t degree_ = 0;
    uint64_t modulus_ = 0, root_ = 0;
};

// ops/fhe_intt/mod.rs:58-160, compute.rs:27-168.
class FheIntt {
public:
    static Result<FheIntt> create(Tensor input, uint32_t degree, uint64_t modulus,
                                  uint64_t inv_root_of_unity);
    Result<Tensor> execute() &&;

private:
    Tensor input_;
    uint32_t degree_ = 0;
    uint64_t modulus_ = 0, inv_root_ = 0;
};

// ops/fhe_pointwise_mul.rs:34-156.
class FhePointwiseMul {
public:
    static Result<FhePointwiseMul> create(Tensor a, Tensor b, uint32_t degree, uint64_t modulus);
    Result<Tensor> execute() const;

private:
    Tensor a_, b_;
    uint32_t degree_ = 0;
    uint64_t modulus_ = 0;
};

// ops/fhe_poly_add.rs:47-175, fhe_poly_sub.rs, fhe_poly_mul.rs: coefficient-
// wise add / sub / mul.  execute() consumes nothing (the Rust ops take self).
enum class CoeffKind { Add, Sub, Mul };
template <CoeffKind K>
class FheCoeffOp {
public:
    static Result<FheCoeffOp> create(Tensor a, Tensor b, uint32_t degree, uint64_t modulus);
    Result<Tensor> execute() const;

private:
    Tensor a_, b_;
    uint32_t degree_ = 0;
    uint64_t modulus_ = 0;
};
using FhePolyAdd = FheCoeffOp<CoeffKind::Add>;
using FhePolySub = FheCoeffOp<CoeffKind::Sub>;
using FhePolyMul = FheCoeffOp<CoeffKind::Mul>;

// ops/fhe_rotate.rs:64-183: Galois automorphism X -> X^(2r+1) of one
// polynomial (negative r counts from degree), coefficients moved to
// i (2r+1) mod 2N and negated as modulus - c (0 stays 0) where that index
// wraps past N.
class FheRotate {
public:
    static Result<FheRotate> create(Tensor input, uint32_t degree, int32_t rotation, uint64_t modulus);
    Result<Tensor> execute() &&;

private:
    Tensor input_;
    uint32_t degree_ = 0;
    int32_t rotation_ = 0;
    uint64_t modulus_ = 0;
};

// ops/fhe_modulus_switch.rs:60-167: round(c * new / old) mod new per
// coefficient, with the product kept exact in 128 bits.
class FheModulusSwitch {
public:
    static Result<FheModulusSwitch> create(Tensor input, uint32_t degree, uint64_t modulus_old,
                                           uint64_t modulus_new);
    Result<Tensor> execute() &&;

private:
    Tensor input_;
    uint32_t degree_ = 0;
    uint64_t modulus_old_ = 0, modulus_new_ = 0;
};

// ops/fhe_key_switch.rs:70-223: validates the decomposition parameters;
// execute() returns a copy of the input, which is what the reference's two
// passes leave in the output (the second one copies the input over the
// first one's digits).
class FheKeySwitch {
public:
    static Result<FheKeySwitch> create(Tensor input, uint32_t degree, uint64_t modulus, uint32_t decomp_base,
                                       uint32_t decomp_levels);
    Result<Tensor> execute() &&;

private:
    Tensor input_;
    uint32_t degree_ = 0;
    uint64_t modulus_ = 0;
    uint32_t decomp_base_ = 0, decomp_levels_ = 0;
};

// ops/fhe_fast_poly_mul.rs:39-171.
class FheFastPolyMul {
public:
    static Result<FheFastPolyMul> create(Tensor a, Tensor b, uint32_t degree, uint64_t modulus,
                                         uint64_t root_of_unity);
    Result<Tensor> execute() const;
    double expected_speedup() const;

private:
    Tensor a_, b_;
    uint32_t degree_ = 0;
    uint64_t modulus_ = 0, root_ = 0;
};

}  // namespace barracuda
