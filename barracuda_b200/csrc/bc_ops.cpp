// bc_ops.cpp -- the reference op API (validation text, execute semantics)
// as C++ classes and as the bc_fhe_* C ABI entry points.
#include "bc_ops.hpp"

#include <cmath>

#include "bc_common.hpp"
#include "bc_runtime.hpp"

namespace bc {
const char *last_error_cstr();
}

using bc::fail;
using bc::format;

namespace {

// ---- validation, in the order and wording of the Rust constructors ----

// FheNtt::new, crates/barracuda/src/ops/fhe_ntt/mod.rs:95-124.
int check_ntt(size_t len_u32, uint32_t degree, uint64_t modulus) {
    const size_t expected = static_cast<size_t>(degree) * 2;
    if (len_u32 != expected)
        return fail(BC_ERR_DEVICE, format("Input length %zu doesn't match expected %zu (degree %u * 2)",
                                          len_u32, expected, degree));
    if (degree < 2 || !bc::is_pow2(degree))
        return fail(BC_ERR_DEVICE, format("Degree %u must be a power of 2 \xE2\x89\xA5 2 for NTT", degree));
    if (modulus == 0) return fail(BC_ERR_DEVICE, "Modulus must be non-zero");
    if ((modulus - 1) % (2ull * degree) != 0)
        return fail(BC_ERR_DEVICE,
                    format("Modulus %llu must satisfy q \xE2\x89\xA1 1 (mod 2N) where N=%u",
                           static_cast<unsigned long long>(modulus), degree));
    return BC_OK;
}

// FheIntt::new, ops/fhe_intt/mod.rs:82-104 (no congruence check, degree 1 allowed).
int check_intt(size_t len_u32, uint32_t degree, uint64_t modulus) {
    const size_t expected = static_cast<size_t>(degree) * 2;
    if (len_u32 != expected)
        return fail(BC_ERR_DEVICE, format("Input length %zu doesn't match expected %zu (degree %u * 2)",
                                          len_u32, expected, degree));
    if (!bc::is_pow2(degree))
        return fail(BC_ERR_DEVICE, format("Degree %u must be a power of 2 for INTT", degree));
    if (modulus == 0) return fail(BC_ERR_DEVICE, "Modulus must be non-zero");
    return BC_OK;
}

// FhePointwiseMul::new (fhe_pointwise_mul.rs:64-92) and FheFastPolyMul::new
// (fhe_fast_poly_mul.rs:61-95) share these checks.
int check_pair(size_t a_len, size_t b_len, uint32_t degree) {
    if (!bc::is_pow2(degree)) return fail(BC_ERR_DEVICE, format("Degree must be power of 2, got %u", degree));
    if (degree < 4 || degree > 65536)
        return fail(BC_ERR_DEVICE, format("Degree must be in range [4, 65_536], got %u", degree));
    const size_t expected = static_cast<size_t>(degree) * 2;
    if (a_len != expected)
        return fail(BC_ERR_DEVICE,
                    format("Input A has wrong length: expected %zu, got %zu", expected, a_len));
    if (b_len != expected)
        return fail(BC_ERR_DEVICE,
                    format("Input B has wrong length: expected %zu, got %zu", expected, b_len));
    return BC_OK;
}

// FhePolyAdd::new (ops/fhe_poly_add.rs:64-101), FhePolySub::new and
// FhePolyMul::new (fhe_poly_sub.rs, fhe_poly_mul.rs:34-66): both lengths,
// then the modulus.  (Their same-device check has no counterpart for raw
// device pointers of one context.)
int check_coeff_lengths(size_t a_len, size_t b_len, uint32_t degree) {
    const size_t expected = static_cast<size_t>(degree) * 2;
    if (a_len != expected)
        return fail(BC_ERR_DEVICE, format("poly_a length %zu doesn't match expected %zu (degree %u * 2)",
                                          a_len, expected, degree));
    if (b_len != expected)
        return fail(BC_ERR_DEVICE, format("poly_b length %zu doesn't match expected %zu (degree %u * 2)",
                                          b_len, expected, degree));
    return BC_OK;
}

int check_coeff(size_t a_len, size_t b_len, uint32_t degree, uint64_t modulus) {
    const int st = check_coeff_lengths(a_len, b_len, degree);
    if (st) return st;
    if (modulus == 0) return fail(BC_ERR_DEVICE, "Modulus must be non-zero");
    return BC_OK;
}

int run_coeff(bc_ctx *ctx, int op, const uint64_t *a, const uint64_t *b, uint32_t degree,
              uint64_t modulus, uint64_t *out) {
    if (degree == 0) return BC_OK;
    if (!a || !b || !out) return fail(BC_ERR_INVALID_INPUT, "device pointers must not be NULL");
    int st = bc::use_device(ctx);
    if (st) return st;
    bc::KArgs k = {};
    k.in = a;
    k.in2 = b;
    k.out = out;
    k.poly_stride = degree;
    k.limb_stride = degree;
    k.batch = 1;
    k.n_limbs = 1;
    k.status = ctx->d_status;
    if ((st = bc::launch_coeff_op(op, k, degree, nullptr, bc::coeff_const(modulus), ctx->stream))) return st;
    return bc::ctx_sync(ctx);
}

// FheRotate::new, FheModulusSwitch::new and FheKeySwitch::new share the
// degree and input-length checks (ops/fhe_rotate.rs:92-113,
// fhe_modulus_switch.rs:86-107, fhe_key_switch.rs:108-139), all InvalidInput.
int check_degree4(uint32_t degree) {
    if (!bc::is_pow2(degree) || degree < 4)
        return fail(BC_ERR_INVALID_INPUT, format("Degree must be power of 2 >= 4, got %u", degree));
    return BC_OK;
}

int check_input_len(size_t len_u32, uint32_t degree) {
    const size_t expected = static_cast<size_t>(degree) * 2;
    if (len_u32 != expected)
        return fail(BC_ERR_INVALID_INPUT,
                    format("Input must have %zu elements (degree=%u, u64 emulated), got %zu", expected, degree,
                           len_u32));
    return BC_OK;
}

// fhe_rotate.rs:92-113.  |rotation| is taken in 64 bits, so INT32_MIN is
// out of range (Rust's i32::abs overflows there).
int check_rotate(size_t len_u32, uint32_t degree, int32_t rotation) {
    int st = check_degree4(degree);
    if (st) return st;
    const int64_t max_rotation = degree / 2;
    const int64_t mag = rotation < 0 ? -static_cast<int64_t>(rotation) : rotation;
    if (mag > max_rotation)
        return fail(BC_ERR_INVALID_INPUT,
                    format("Rotation %d out of range [-%lld, %lld] for degree %u", rotation,
                           static_cast<long long>(max_rotation), static_cast<long long>(max_rotation), degree));
    return check_input_len(len_u32, degree);
}

// fhe_modulus_switch.rs:86-107.
int check_modulus_switch(size_t len_u32, uint32_t degree, uint64_t modulus_old, uint64_t modulus_new) {
    int st = check_degree4(degree);
    if (st) return st;
    if (modulus_new >= modulus_old)
        return fail(BC_ERR_INVALID_INPUT, format("New modulus (%llu) must be < old modulus (%llu)",
                                                 static_cast<unsigned long long>(modulus_new),
                                                 static_cast<unsigned long long>(modulus_old)));
    return check_input_len(len_u32, degree);
}

// fhe_key_switch.rs:108-139.
int check_key_switch(size_t len_u32, uint32_t degree, uint32_t decomp_base, uint32_t decomp_levels) {
    int st = check_degree4(degree);
    if (st) return st;
    if (decomp_base < 2 || decomp_base > (1u << 24))
        return fail(BC_ERR_INVALID_INPUT, format("Decomposition base must be in [2, 2^24], got %u", decomp_base));
    if (decomp_levels == 0 || decomp_levels > 32)
        return fail(BC_ERR_INVALID_INPUT, format("Decomposition levels must be in [1, 32], got %u", decomp_levels));
    return check_input_len(len_u32, degree);
}

// fhe_rotate.rs:150-155: rotation normalised into [0, degree), galois 2r + 1.
uint32_t rotate_galois(uint32_t degree, int32_t rotation) {
    const uint32_t r = rotation < 0 ? static_cast<uint32_t>(static_cast<int64_t>(degree) + rotation)
                                    : static_cast<uint32_t>(rotation);
    return 2u * r + 1u;
}

int run_rotate(bc_ctx *ctx, const uint64_t *in, uint32_t degree, int32_t rotation, uint64_t modulus,
               uint64_t *out) {
    if (!in || !out) return fail(BC_ERR_INVALID_INPUT, "device pointers must not be NULL");
    if (in == out) return fail(BC_ERR_INVALID_INPUT, "input and output must be different buffers");
    int st = bc::use_device(ctx);
    if (st) return st;
    bc::KArgs k = {};
    k.in = in;
    k.out = out;
    k.poly_stride = degree;
    k.limb_stride = degree;
    k.batch = 1;
    k.n_limbs = 1;
    k.logn = bc::ilog2(degree);
    k.status = ctx->d_status;
    if ((st = bc::launch_automorphism(k, rotate_galois(degree, rotation), nullptr, modulus, ctx->stream)))
        return st;
    return bc::ctx_sync(ctx);
}

int run_modulus_switch(bc_ctx *ctx, const uint64_t *in, uint32_t degree, uint64_t modulus_old,
                       uint64_t modulus_new, uint64_t *out) {
    if (!in || !out) return fail(BC_ERR_INVALID_INPUT, "device pointers must not be NULL");
    int st = bc::use_device(ctx);
    if (st) return st;
    if ((st = bc::launch_modulus_switch(in, out, degree, bc::modswitch_const(modulus_old, modulus_new),
                                        ctx->stream)))
        return st;
    return bc::ctx_sync(ctx);
}

// FheKeySwitch::execute's second pass stores the input over the first
// pass's digits (fhe_key_switch.wgsl:128-148 reads binding 0, the input), so
// the op's result is a copy of its input.
int run_key_switch(bc_ctx *ctx, const uint64_t *in, uint32_t degree, uint64_t *out) {
    if (!in || !out) return fail(BC_ERR_INVALID_INPUT, "device pointers must not be NULL");
    int st = bc::use_device(ctx);
    if (st) return st;
    if (in != out) {
        const cudaError_t e = cudaMemcpyAsync(out, in, static_cast<size_t>(degree) * sizeof(uint64_t),
                                              cudaMemcpyDeviceToDevice, ctx->stream);
        if (e != cudaSuccess) return bc::cuda_fail(e, "key switch copy");
    }
    return bc::ctx_sync(ctx);
}

// Moduli the CUDA path cannot represent (>= 2^62): the reference accepts
// them but computes truncated products there.
int check_width(uint64_t modulus) {
    if (modulus >= (1ull << 62))
        return fail(BC_ERR_UNSUPPORTED,
                    format("modulus %llu is >= 2^62; the CUDA path supports moduli below 2^62",
                           static_cast<unsigned long long>(modulus)));
    return BC_OK;
}

int run_ntt(bc_ctx *ctx, const uint64_t *in, uint32_t degree, uint64_t modulus, uint64_t root,
            uint64_t *out) {
    int st = check_width(modulus);
    if (st) return st;
    std::shared_ptr<bc_plan> sp;
    if ((st = bc::cached_plan(ctx, degree, modulus, root, 0, BC_NTT_CYCLIC, &sp))) return st;
    if ((st = bc::run_forward(sp.get(), in, out, 1, nullptr, ctx->stream))) return st;
    return bc::ctx_sync(ctx);
}

int run_intt(bc_ctx *ctx, const uint64_t *in, uint32_t degree, uint64_t modulus, uint64_t inv_root,
             uint64_t *out) {
    int st = check_width(modulus);
    if (st) return st;
    std::shared_ptr<bc_plan> sp;
    // cyclic plan whose inverse table is built from inv_root
    if ((st = bc::cached_plan(ctx, degree, modulus, 0, inv_root, BC_NTT_CYCLIC, &sp))) return st;
    if ((st = bc::run_inverse(sp.get(), in, out, 1, nullptr, ctx->stream))) return st;
    return bc::ctx_sync(ctx);
}

int run_pointwise(bc_ctx *ctx, const uint64_t *a, const uint64_t *b, uint32_t degree,
                  uint64_t modulus, uint64_t *out) {
    int st;
    if (modulus == 0) {
        // The reference constructor accepts q = 0 and its shader then keeps
        // the low 32 bits of each product (fhe_pointwise_mul.wgsl:70-95).
        if ((st = bc::use_device(ctx))) return st;
        bc::KArgs k = {};
        k.in = a;
        k.in2 = b;
        k.out = out;
        k.poly_stride = degree;
        k.limb_stride = degree;
        k.batch = 1;
        k.n_limbs = 1;
        k.logn = bc::ilog2(degree);
        k.status = ctx->d_status;
        if ((st = bc::launch_mul_lo32(k, ctx->stream))) return st;
        return bc::ctx_sync(ctx);
    }
    if ((st = check_width(modulus))) return st;
    std::shared_ptr<bc_plan> sp;
    if ((st = bc::cached_plan(ctx, degree, modulus, 0, 0, BC_NTT_CYCLIC, &sp))) return st;
    if ((st = bc::run_pointwise(sp.get(), a, b, out, 1, nullptr, ctx->stream))) return st;
    return bc::ctx_sync(ctx);
}

int run_fast_poly_mul(bc_ctx *ctx, const uint64_t *a, const uint64_t *b, uint32_t degree,
                      uint64_t modulus, uint64_t root, uint64_t *out) {
    // execute() builds FheNtt for both inputs first (fhe_fast_poly_mul.rs:124-139),
    // so the NTT constructor's modulus checks apply here.
    int st = check_ntt(static_cast<size_t>(degree) * 2, degree, modulus);
    if (st) return st;
    if ((st = check_width(modulus))) return st;
    const uint64_t inv_root = bc::ref_fastmul_modinv(root, modulus);
    std::shared_ptr<bc_plan> sp;
    if ((st = bc::cached_plan(ctx, degree, modulus, root, inv_root, BC_NTT_CYCLIC, &sp))) return st;
    if ((st = bc::run_polymul(sp.get(), a, b, out, 1, nullptr, ctx->stream))) return st;
    return bc::ctx_sync(ctx);
}

}  // namespace

// ================================================================ C++ API

namespace barracuda {

namespace {
Error last(int st) { return Error{st, bc::last_error_cstr()}; }
}  // namespace

std::string Error::to_string() const {
    switch (kind) {
    case BC_ERR_DEVICE: return "Device error: " + message;
    case BC_ERR_INVALID_INPUT: return "Invalid input: " + message;
    case BC_ERR_OUT_OF_MEMORY: return "Out of memory: " + message;
    case BC_ERR_DEVICE_LOST: return "GPU device lost: " + message;
    case BC_ERR_GPU: return "GPU error: " + message;
    case BC_ERR_UNSUPPORTED: return "Operation not supported on device: " + message;
    case BC_ERR_DEVICE_NOT_AVAILABLE: return "Device not available: " + message;
    case BC_ERR_EXECUTION: return "Execution error: " + message;
    case BC_ERR_INTERNAL: return "Internal error: " + message;
    default: return message;
    }
}

Result<std::shared_ptr<Device>> Device::open(int ordinal) {
    bc_ctx *c = nullptr;
    const int st = bc_ctx_create(ordinal, &c);
    if (st) return Result<std::shared_ptr<Device>>::err(last(st));
    return Result<std::shared_ptr<Device>>::ok(std::shared_ptr<Device>(new Device(c)));
}

Device::~Device() { bc_ctx_destroy(ctx_); }

Result<Tensor> Tensor::empty_u64(size_t n_u64, std::shared_ptr<Device> dev) {
    void *p = nullptr;
    const int st = bc_buf_alloc(dev->ctx(), n_u64 * 8, &p);
    if (st) return Result<Tensor>::err(last(st));
    Tensor t;
    bc_ctx *c = dev->ctx();
    t.dev_ = dev;
    t.buf_ = std::shared_ptr<void>(p, [dev](void *q) { bc_buf_free(dev->ctx(), q); });
    t.len_u32_ = n_u64 * 2;
    (void)c;
    return Result<Tensor>::ok(std::move(t));
}

Result<Tensor> Tensor::from_u32(const std::vector<uint32_t> &data, std::shared_ptr<Device> dev) {
    auto r = empty_u64((data.size() + 1) / 2, dev);
    if (r.is_err()) return r;
    Tensor t = r.take();
    t.len_u32_ = data.size();
    const int st = bc_buf_h2d(dev->ctx(), t.mutable_data(), data.data(), data.size() * 4);
    if (st) return Result<Tensor>::err(last(st));
    return Result<Tensor>::ok(std::move(t));
}

Result<std::vector<uint32_t>> Tensor::to_vec_u32() const {
    std::vector<uint32_t> out(len_u32_);
    const int st = bc_buf_d2h(dev_->ctx(), out.data(), buf_.get(), len_u32_ * 4);
    if (st) return Result<std::vector<uint32_t>>::err(last(st));
    return Result<std::vector<uint32_t>>::ok(std::move(out));
}

Result<Tensor> create_fhe_poly_tensor(const std::vector<uint64_t> &poly, std::shared_ptr<Device> dev) {
    std::vector<uint32_t> words;
    words.reserve(poly.size() * 2);
    for (uint64_t v : poly) {
        words.push_back(static_cast<uint32_t>(v));
        words.push_back(static_cast<uint32_t>(v >> 32));
    }
    return Tensor::from_u32(words, std::move(dev));
}

uint64_t compute_primitive_root(uint32_t degree, uint64_t modulus) {
    return bc_compute_primitive_root(degree, modulus);
}

uint64_t compute_inverse_root(uint32_t degree, uint64_t modulus, uint64_t root) {
    return bc_compute_inverse_root(degree, modulus, root);
}

Result<FheNtt> FheNtt::create(Tensor input, uint32_t degree, uint64_t modulus, uint64_t root) {
    const int st = check_ntt(input.len(), degree, modulus);
    if (st) return Result<FheNtt>::err(last(st));
    FheNtt op;
    op.input_ = std::move(input);
    op.degree_ = degree;
    op.modulus_ = modulus;
    op.root_ = root;
    return Result<FheNtt>::ok(std::move(op));
}

Result<Tensor> FheNtt::execute() && {
    auto out = Tensor::empty_u64(degree_, input_.device());
    if (out.is_err()) return out;
    const int st = run_ntt(input_.device()->ctx(), input_.data(), degree_, modulus_, root_,
                           out.value().mutable_data());
    if (st) return Result<Tensor>::err(last(st));
    return out;
}

Result<FheIntt> FheIntt::create(Tensor input, uint32_t degree, uint64_t modulus, uint64_t inv_root) {
    const int st = check_intt(input.len(), degree, modulus);
    if (st) return Result<FheIntt>::err(last(st));
    FheIntt op;
    op.input_ = std::move(input);
    op.degree_ = degree;
    op.modulus_ = modulus;
    op.inv_root_ = inv_root;
    return Result<FheIntt>::ok(std::move(op));
}

Result<Tensor> FheIntt::execute() && {
    auto out = Tensor::empty_u64(degree_, input_.device());
    if (out.is_err()) return out;
    const int st = run_intt(input_.device()->ctx(), input_.data(), degree_, modulus_, inv_root_,
                            out.value().mutable_data());
    if (st) return Result<Tensor>::err(last(st));
    return out;
}

Result<FhePointwiseMul> FhePointwiseMul::create(Tensor a, Tensor b, uint32_t degree, uint64_t modulus) {
    int st = check_pair(a.len(), b.len(), degree);
    if (!st && a.device() != b.device())
        st = fail(BC_ERR_DEVICE, "input_a and input_b must be on the same device");
    if (st) return Result<FhePointwiseMul>::err(last(st));
    FhePointwiseMul op;
    op.a_ = std::move(a);
    op.b_ = std::move(b);
    op.degree_ = degree;
    op.modulus_ = modulus;
    return Result<FhePointwiseMul>::ok(std::move(op));
}

Result<Tensor> FhePointwiseMul::execute() const {
    auto out = Tensor::empty_u64(degree_, a_.device());
    if (out.is_err()) return out;
    const int st = run_pointwise(a_.device()->ctx(), a_.data(), b_.data(), degree_, modulus_,
                                 out.value().mutable_data());
    if (st) return Result<Tensor>::err(last(st));
    return out;
}

template <CoeffKind K>
Result<FheCoeffOp<K>> FheCoeffOp<K>::create(Tensor a, Tensor b, uint32_t degree, uint64_t modulus) {
    int st = check_coeff_lengths(a.len(), b.len(), degree);
    if (!st && a.device() != b.device()) st = fail(BC_ERR_DEVICE, "poly_a and poly_b must be on the same device");
    if (!st && modulus == 0) st = fail(BC_ERR_DEVICE, "Modulus must be non-zero");
    if (st) return Result<FheCoeffOp>::err(last(st));
    FheCoeffOp op;
    op.a_ = std::move(a);
    op.b_ = std::move(b);
    op.degree_ = degree;
    op.modulus_ = modulus;
    return Result<FheCoeffOp>::ok(std::move(op));
}

template <CoeffKind K>
Result<Tensor> FheCoeffOp<K>::execute() const {
    auto out = Tensor::empty_u64(degree_, a_.device());
    if (out.is_err()) return out;
    const int op = K == CoeffKind::Add ? bc::kCoeffAdd : K == CoeffKind::Sub ? bc::kCoeffSub : bc::kCoeffMul;
    const int st = run_coeff(a_.device()->ctx(), op, a_.data(), b_.data(), degree_, modulus_,
                             out.value().mutable_data());
    if (st) return Result<Tensor>::err(last(st));
    return out;
}

template class FheCoeffOp<CoeffKind::Add>;
template class FheCoeffOp<CoeffKind::Sub>;
template class FheCoeffOp<CoeffKind::Mul>;

Result<FheRotate> FheRotate::create(Tensor input, uint32_t degree, int32_t rotation, uint64_t modulus) {
    const int st = check_rotate(input.len(), degree, rotation);
    if (st) return Result<FheRotate>::err(last(st));
    FheRotate op;
    op.input_ = std::move(input);
    op.degree_ = degree;
    op.rotation_ = rotation;
    op.modulus_ = modulus;
    return Result<FheRotate>::ok(std::move(op));
}

Result<Tensor> FheRotate::execute() && {
    auto out = Tensor::empty_u64(degree_, input_.device());
    if (out.is_err()) return out;
    const int st = run_rotate(input_.device()->ctx(), input_.data(), degree_, rotation_, modulus_,
                              out.value().mutable_data());
    if (st) return Result<Tensor>::err(last(st));
    return out;
}

Result<FheModulusSwitch> FheModulusSwitch::create(Tensor input, uint32_t degree, uint64_t modulus_old,
                                                  uint64_t modulus_new) {
    const int st = check_modulus_switch(input.len(), degree, modulus_old, modulus_new);
    if (st) return Result<FheModulusSwitch>::err(last(st));
    FheModulusSwitch op;
    op.input_ = std::move(input);
    op.degree_ = degree;
    op.modulus_old_ = modulus_old;
    op.modulus_new_ = modulus_new;
    return Result<FheModulusSwitch>::ok(std::move(op));
}

Result<Tensor> FheModulusSwitch::execute() && {
    auto out = Tensor::empty_u64(degree_, input_.device());
    if (out.is_err()) return out;
    const int st = run_modulus_switch(input_.device()->ctx(), input_.data(), degree_, modulus_old_, modulus_new_,
                                      out.value().mutable_data());
    if (st) return Result<Tensor>::err(last(st));
    return out;
}

Result<FheKeySwitch> FheKeySwitch::create(Tensor input, uint32_t degree, uint64_t modulus, uint32_t decomp_base,
                                          uint32_t decomp_levels) {
    const int st = check_key_switch(input.len(), degree, decomp_base, decomp_levels);
    if (st) return Result<FheKeySwitch>::err(last(st));
    FheKeySwitch op;
    op.input_ = std::move(input);
    op.degree_ = degree;
    op.modulus_ = modulus;
    op.decomp_base_ = decomp_base;
    op.decomp_levels_ = decomp_levels;
    return Result<FheKeySwitch>::ok(std::move(op));
}

Result<Tensor> FheKeySwitch::execute() && {
    auto out = Tensor::empty_u64(degree_, input_.device());
    if (out.is_err()) return out;
    const int st = run_key_switch(input_.device()->ctx(), input_.data(), degree_, out.value().mutable_data());
    if (st) return Result<Tensor>::err(last(st));
    return out;
}

Result<FheFastPolyMul> FheFastPolyMul::create(Tensor a, Tensor b, uint32_t degree, uint64_t modulus,
                                              uint64_t root) {
    const int st = check_pair(a.len(), b.len(), degree);
    if (st) return Result<FheFastPolyMul>::err(last(st));
    FheFastPolyMul op;
    op.a_ = std::move(a);
    op.b_ = std::move(b);
    op.degree_ = degree;
    op.modulus_ = modulus;
    op.root_ = root;
    return Result<FheFastPolyMul>::ok(std::move(op));
}

Result<Tensor> FheFastPolyMul::execute() const {
    auto out = Tensor::empty_u64(degree_, a_.device());
    if (out.is_err()) return out;
    const int st = run_fast_poly_mul(a_.device()->ctx(), a_.data(), b_.data(), degree_, modulus_,
                                     root_, out.value().mutable_data());
    if (st) return Result<Tensor>::err(last(st));
    return out;
}

// fhe_fast_poly_mul.rs:160-170: N / log2 N times the 16.4% efficiency the
// reference measured for its own path.
double FheFastPolyMul::expected_speedup() const {
    const double n = static_cast<double>(degree_);
    return n / std::log2(n) * 0.164;
}

}  // namespace barracuda

// ================================================================== C ABI

extern "C" {

uint64_t bc_compute_primitive_root(uint32_t degree, uint64_t modulus) {
    return bc::ref_primitive_root(degree, modulus);
}

uint64_t bc_compute_inverse_root(uint32_t degree, uint64_t modulus, uint64_t root) {
    (void)degree;
    return bc::ref_modinv(root, modulus);
}

int bc_fhe_ntt_check(size_t input_len_u32, uint32_t degree, uint64_t modulus, uint64_t root) {
    (void)root;
    return check_ntt(input_len_u32, degree, modulus);
}

int bc_fhe_ntt(bc_ctx *ctx, const uint64_t *d_in, size_t input_len_u32, uint32_t degree,
               uint64_t modulus, uint64_t root, uint64_t *d_out) {
    if (!ctx) return fail(BC_ERR_INVALID_INPUT, "NULL context");
    const int st = check_ntt(input_len_u32, degree, modulus);
    return st ? st : run_ntt(ctx, d_in, degree, modulus, root, d_out);
}

int bc_fhe_intt_check(size_t input_len_u32, uint32_t degree, uint64_t modulus, uint64_t inv_root) {
    (void)inv_root;
    return check_intt(input_len_u32, degree, modulus);
}

int bc_fhe_intt(bc_ctx *ctx, const uint64_t *d_in, size_t input_len_u32, uint32_t degree,
                uint64_t modulus, uint64_t inv_root, uint64_t *d_out) {
    if (!ctx) return fail(BC_ERR_INVALID_INPUT, "NULL context");
    const int st = check_intt(input_len_u32, degree, modulus);
    return st ? st : run_intt(ctx, d_in, degree, modulus, inv_root, d_out);
}

int bc_fhe_pointwise_mul_check(size_t a_len_u32, size_t b_len_u32, uint32_t degree, uint64_t modulus) {
    (void)modulus;
    return check_pair(a_len_u32, b_len_u32, degree);
}

int bc_fhe_pointwise_mul(bc_ctx *ctx, const uint64_t *d_a, size_t a_len_u32, const uint64_t *d_b,
                         size_t b_len_u32, uint32_t degree, uint64_t modulus, uint64_t *d_out) {
    if (!ctx) return fail(BC_ERR_INVALID_INPUT, "NULL context");
    const int st = check_pair(a_len_u32, b_len_u32, degree);
    return st ? st : run_pointwise(ctx, d_a, d_b, degree, modulus, d_out);
}

int bc_fhe_fast_poly_mul_check(size_t a_len_u32, size_t b_len_u32, uint32_t degree, uint64_t modulus,
                               uint64_t root) {
    (void)modulus;
    (void)root;
    return check_pair(a_len_u32, b_len_u32, degree);
}

int bc_fhe_fast_poly_mul(bc_ctx *ctx, const uint64_t *d_a, size_t a_len_u32, const uint64_t *d_b,
                         size_t b_len_u32, uint32_t degree, uint64_t modulus, uint64_t root,
                         uint64_t *d_out) {
    if (!ctx) return fail(BC_ERR_INVALID_INPUT, "NULL context");
    const int st = check_pair(a_len_u32, b_len_u32, degree);
    return st ? st : run_fast_poly_mul(ctx, d_a, d_b, degree, modulus, root, d_out);
}

int bc_fhe_poly_add_check(size_t a_len_u32, size_t b_len_u32, uint32_t degree, uint64_t modulus) {
    return check_coeff(a_len_u32, b_len_u32, degree, modulus);
}
int bc_fhe_poly_sub_check(size_t a_len_u32, size_t b_len_u32, uint32_t degree, uint64_t modulus) {
    return check_coeff(a_len_u32, b_len_u32, degree, modulus);
}
int bc_fhe_poly_mul_check(size_t a_len_u32, size_t b_len_u32, uint32_t degree, uint64_t modulus) {
    return check_coeff(a_len_u32, b_len_u32, degree, modulus);
}

static int coeff_entry(int op, bc_ctx *ctx, const uint64_t *d_a, size_t a_len, const uint64_t *d_b,
                       size_t b_len, uint32_t degree, uint64_t modulus, uint64_t *d_out) {
    if (!ctx) return fail(BC_ERR_INVALID_INPUT, "NULL context");
    const int st = check_coeff(a_len, b_len, degree, modulus);
    return st ? st : run_coeff(ctx, op, d_a, d_b, degree, modulus, d_out);
}

int bc_fhe_poly_add(bc_ctx *ctx, const uint64_t *d_a, size_t a_len_u32, const uint64_t *d_b,
                    size_t b_len_u32, uint32_t degree, uint64_t modulus, uint64_t *d_out) {
    return coeff_entry(bc::kCoeffAdd, ctx, d_a, a_len_u32, d_b, b_len_u32, degree, modulus, d_out);
}
int bc_fhe_poly_sub(bc_ctx *ctx, const uint64_t *d_a, size_t a_len_u32, const uint64_t *d_b,
                    size_t b_len_u32, uint32_t degree, uint64_t modulus, uint64_t *d_out) {
    return coeff_entry(bc::kCoeffSub, ctx, d_a, a_len_u32, d_b, b_len_u32, degree, modulus, d_out);
}
int bc_fhe_poly_mul(bc_ctx *ctx, const uint64_t *d_a, size_t a_len_u32, const uint64_t *d_b,
                    size_t b_len_u32, uint32_t degree, uint64_t modulus, uint64_t *d_out) {
    return coeff_entry(bc::kCoeffMul, ctx, d_a, a_len_u32, d_b, b_len_u32, degree, modulus, d_out);
}

int bc_fhe_rotate_check(size_t input_len_u32, uint32_t degree, int32_t rotation, uint64_t modulus) {
    (void)modulus;
    return check_rotate(input_len_u32, degree, rotation);
}

int bc_fhe_rotate(bc_ctx *ctx, const uint64_t *d_in, size_t input_len_u32, uint32_t degree, int32_t rotation,
                  uint64_t modulus, uint64_t *d_out) {
    if (!ctx) return fail(BC_ERR_INVALID_INPUT, "NULL context");
    const int st = check_rotate(input_len_u32, degree, rotation);
    return st ? st : run_rotate(ctx, d_in, degree, rotation, modulus, d_out);
}

int bc_fhe_modulus_switch_check(size_t input_len_u32, uint32_t degree, uint64_t modulus_old,
                                uint64_t modulus_new) {
    return check_modulus_switch(input_len_u32, degree, modulus_old, modulus_new);
}

int bc_fhe_modulus_switch(bc_ctx *ctx, const uint64_t *d_in, size_t input_len_u32, uint32_t degree,
                          uint64_t modulus_old, uint64_t modulus_new, uint64_t *d_out) {
    if (!ctx) return fail(BC_ERR_INVALID_INPUT, "NULL context");
    const int st = check_modulus_switch(input_len_u32, degree, modulus_old, modulus_new);
    return st ? st : run_modulus_switch(ctx, d_in, degree, modulus_old, modulus_new, d_out);
}

int bc_fhe_key_switch_check(size_t input_len_u32, uint32_t degree, uint64_t modulus, uint32_t decomp_base,
                            uint32_t decomp_levels) {
    (void)modulus;
    return check_key_switch(input_len_u32, degree, decomp_base, decomp_levels);
}

int bc_fhe_key_switch(bc_ctx *ctx, const uint64_t *d_in, size_t input_len_u32, uint32_t degree, uint64_t modulus,
                      uint32_t decomp_base, uint32_t decomp_levels, uint64_t *d_out) {
    (void)modulus;
    if (!ctx) return fail(BC_ERR_INVALID_INPUT, "NULL context");
    const int st = check_key_switch(input_len_u32, degree, decomp_base, decomp_levels);
    return st ? st : run_key_switch(ctx, d_in, degree, d_out);
}

uint32_t bc_rotation_galois(uint32_t degree, int32_t rotation) {
    if (check_rotate(static_cast<size_t>(degree) * 2, degree, rotation)) return 0;
    return rotate_galois(degree, rotation);
}

}  // extern "C"
