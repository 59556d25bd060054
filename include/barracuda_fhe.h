/*
 * barracuda_fhe.h -- C ABI of the B200-native FHE NTT path.
 *
 * The shared library libbarracuda_fhe.so implements barraCuda's FHE hot path
 * (forward NTT, inverse INTT, pointwise modular multiply, NTT-based
 * polynomial product) with hand-written sm_100a CUDA kernels.  The ABI uses
 * plain pointers, sizes and integer status codes only, so that a thin Rust
 * crate (barracuda-cuda-sys) can bind it with `extern "C"` declarations and
 * keep every `unsafe` block in that one crate.
 *
 * Reference interfaces replaced (paths inside ecoPrimals/barraCuda):
 *   - crates/barracuda/src/ops/fhe_ntt/mod.rs:95 FheNtt::new,
 *     fhe_ntt/compute.rs:29 FheNtt::execute                 -> bc_fhe_ntt*
 *   - ops/fhe_intt/mod.rs:82 FheIntt::new, compute.rs:27     -> bc_fhe_intt*
 *   - ops/fhe_pointwise_mul.rs:64,119 FhePointwiseMul        -> bc_fhe_pointwise_mul*
 *   - ops/fhe_fast_poly_mul.rs:61,122 FheFastPolyMul         -> bc_fhe_fast_poly_mul*
 *   - ops/fhe_poly_add.rs:64,128 FhePolyAdd, fhe_poly_sub.rs FhePolySub,
 *     fhe_poly_mul.rs:34,82 FhePolyMul                       -> bc_fhe_poly_{add,sub,mul}*
 *   - ops/fhe_rotate.rs:91,140 FheRotate                     -> bc_fhe_rotate*
 *   - ops/fhe_modulus_switch.rs:85,124 FheModulusSwitch       -> bc_fhe_modulus_switch*
 *   - ops/fhe_key_switch.rs:101,162 FheKeySwitch              -> bc_fhe_key_switch*
 *   - ops/fhe_ntt/mod.rs:210 compute_primitive_root          -> bc_compute_primitive_root
 *   - ops/fhe_intt/mod.rs:202 compute_inverse_root           -> bc_compute_inverse_root
 *   - ops/fhe_poly_add.rs:185 create_fhe_poly_tensor,
 *     tensor/mod.rs:197 Tensor::from_data_pod, :456 to_vec_u32 -> bc_buf_*
 *   - device/backend.rs:311 GpuBackend::dispatch_compute (the per-stage
 *     dispatch the ops issue today)                         -> bc_ntt_* on a plan
 *   - multi_gpu/gpu_pool.rs:194 GpuPool::parallel_map (nearest analog of the
 *     shard split)                                          -> bc_partition
 *
 * Data layout: a polynomial of degree N is N little-endian uint64_t
 * coefficients in natural order, byte-identical to the reference's
 * [lo32, hi32] u32-pair tensors (Tensor::len() == 2N u32 words).
 *
 * Errors: every call returns a bc_status; on failure a message is kept per
 * thread and returned by bc_last_error().  Status codes map one to one onto
 * BarracudaError variants (crates/barracuda/src/error.rs).
 *
 * Threading: one bc_ctx per GPU.  A bc_plan is immutable after creation and
 * may be shared by threads; launches on one stream are ordered.
 */
#ifndef BARRACUDA_FHE_H
#define BARRACUDA_FHE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BC_ABI_VERSION 1

typedef enum bc_status {
    BC_OK = 0,
    BC_ERR_DEVICE = 1,               /* BarracudaError::Device(String), error.rs:20 (op validation) */
    BC_ERR_INVALID_INPUT = 2,        /* BarracudaError::InvalidInput, error.rs:80 */
    BC_ERR_OUT_OF_MEMORY = 3,        /* BarracudaError::OutOfMemory, error.rs:67 */
    BC_ERR_DEVICE_LOST = 4,          /* BarracudaError::DeviceLost, error.rs:59 */
    BC_ERR_GPU = 5,                  /* BarracudaError::Gpu, error.rs:50 */
    BC_ERR_UNSUPPORTED = 6,          /* BarracudaError::UnsupportedOperation, error.rs:71 */
    BC_ERR_DEVICE_NOT_AVAILABLE = 7, /* BarracudaError::DeviceNotAvailable, error.rs:93 */
    BC_ERR_EXECUTION = 8,            /* BarracudaError::ExecutionError, error.rs:86 */
    BC_ERR_INTERNAL = 9              /* BarracudaError::Internal, error.rs:108 */
} bc_status;

typedef struct bc_ctx bc_ctx;
typedef struct bc_plan bc_plan;

/* ---------------------------------------------------------------- basics */

/* Message of the last failed call on this thread ("" if none). */
const char *bc_last_error(void);
int bc_abi_version(void);
int bc_device_count(int *count);

/* One context per GPU: owns a non-blocking stream, a plan cache and a small
 * device status word used by kernels to report bad inputs.
 * Replaces WgpuDevice creation (device/wgpu_device/). */
int bc_ctx_create(int device, bc_ctx **out);
int bc_ctx_destroy(bc_ctx *ctx);
int bc_ctx_device(const bc_ctx *ctx, int *device);
/* cudaStream_t of the context, as void*. */
int bc_ctx_stream(bc_ctx *ctx, void **stream);
/* Waits for the context stream, then reports (and clears) any status a
 * kernel raised since the last check (e.g. a coefficient >= 2^32 given to a
 * plan whose modulus is below 2^31 -> BC_ERR_INVALID_INPUT).
 *
 * Which call an input-range error belongs to: kernels raise the status on
 * the context they were launched for, from any stream, and the next
 * bc_ctx_sync on that context reports it.  The synchronous reference-op
 * calls (bc_fhe_*) sync before they return, so their own bad input fails
 * that call.  The batched plan calls (bc_ntt_*, bc_polymul, ...) are
 * asynchronous: a bad input in one of them is reported by the first
 * bc_ctx_sync after its kernels ran, which names no call.  A caller that
 * must attribute the error syncs after each batched call it wants checked
 * (or keeps inputs below q, the reference's own domain, where no status is
 * ever raised).  The kernels still finish: words >= 2^32 are taken modulo
 * 2^32, so the outputs of a flagged call are not meaningful. */
int bc_ctx_sync(bc_ctx *ctx);

/* --------------------------------------------------------------- buffers */

/* Device memory owned by the caller; synchronous copies use the ctx stream.
 * bc_buf_alloc takes the memory from the context's pool (freed buffers are
 * reused without a driver allocation) and returns it ready for every
 * stream; bc_buf_free waits for all work on the device, as cudaFree does,
 * then returns the memory to the pool. */
int bc_buf_alloc(bc_ctx *ctx, size_t bytes, void **dptr);
int bc_buf_free(bc_ctx *ctx, void *dptr);
int bc_buf_h2d(bc_ctx *ctx, void *dst, const void *src, size_t bytes);
int bc_buf_d2h(bc_ctx *ctx, void *dst, const void *src, size_t bytes);
int bc_buf_h2d_async(bc_ctx *ctx, void *dst, const void *src, size_t bytes, void *stream);
int bc_buf_d2h_async(bc_ctx *ctx, void *dst, const void *src, size_t bytes, void *stream);
/* Page-locked host memory for the async copies above. */
int bc_host_alloc(size_t bytes, void **hptr);
int bc_host_free(void *hptr);

/* ------------------------------------------- reference op API (synchronous)
 * Each pair is <Op>::new validation (the *_check call: same conditions, same
 * order, same message text as the Rust constructor) and <Op>::execute (runs
 * on the context stream and returns after the result is complete, as the
 * reference's submit + poll does).  Lengths are in u32 words, as
 * Tensor::len() reports them.  Outputs are caller-allocated (N u64). */

/* fhe_ntt/mod.rs:210-242 (same candidate order and fallbacks). */
uint64_t bc_compute_primitive_root(uint32_t degree, uint64_t modulus);
/* fhe_intt/mod.rs:202-204 (extended Euclid; 0 if not invertible). */
uint64_t bc_compute_inverse_root(uint32_t degree, uint64_t modulus, uint64_t root);

/* fhe_ntt/mod.rs:95-140 / compute.rs:29-143.  Cyclic DIT transform with the
 * N-th root omega, natural-order output, X_k = sum_j x_j omega^{jk}. */
int bc_fhe_ntt_check(size_t input_len_u32, uint32_t degree, uint64_t modulus,
                     uint64_t root_of_unity);
int bc_fhe_ntt(bc_ctx *ctx, const uint64_t *d_in, size_t input_len_u32, uint32_t degree,
               uint64_t modulus, uint64_t root_of_unity, uint64_t *d_out);

/* fhe_intt/mod.rs:82-124 / compute.rs:27-168.  DIT with the given inverse
 * root, then multiplication by N^-1 (0 when N is not invertible mod q). */
int bc_fhe_intt_check(size_t input_len_u32, uint32_t degree, uint64_t modulus,
                      uint64_t inv_root_of_unity);
int bc_fhe_intt(bc_ctx *ctx, const uint64_t *d_in, size_t input_len_u32, uint32_t degree,
                uint64_t modulus, uint64_t inv_root_of_unity, uint64_t *d_out);

/* fhe_pointwise_mul.rs:64-155.  C[i] = A[i] * B[i] mod q. */
int bc_fhe_pointwise_mul_check(size_t a_len_u32, size_t b_len_u32, uint32_t degree,
                               uint64_t modulus);
int bc_fhe_pointwise_mul(bc_ctx *ctx, const uint64_t *d_a, size_t a_len_u32,
                         const uint64_t *d_b, size_t b_len_u32, uint32_t degree,
                         uint64_t modulus, uint64_t *d_out);

/* fhe_fast_poly_mul.rs:61-154.  INTT(NTT(a) * NTT(b)), fused in one kernel. */
int bc_fhe_fast_poly_mul_check(size_t a_len_u32, size_t b_len_u32, uint32_t degree,
                               uint64_t modulus, uint64_t root_of_unity);
int bc_fhe_fast_poly_mul(bc_ctx *ctx, const uint64_t *d_a, size_t a_len_u32,
                         const uint64_t *d_b, size_t b_len_u32, uint32_t degree,
                         uint64_t modulus, uint64_t root_of_unity, uint64_t *d_out);

/* ops/fhe_poly_add.rs:64-175, fhe_poly_sub.rs, fhe_poly_mul.rs:34-133:
 * coefficient-wise C = A + B, A - B, A * B modulo q (any degree; same checks
 * and message text as the Rust constructors).  Add and sub reproduce the
 * reference bit for bit for any u64 inputs (a wrapping sum minus q at most
 * twice; a - b, or (q - b) + a when a < b).  Mul returns the exact residue
 * (a * b) mod q; the reference's shader matches it only while its product
 * stays below 1001 q and its 32x32 partial products do not overflow. */
int bc_fhe_poly_add_check(size_t a_len_u32, size_t b_len_u32, uint32_t degree, uint64_t modulus);
int bc_fhe_poly_add(bc_ctx *ctx, const uint64_t *d_a, size_t a_len_u32, const uint64_t *d_b,
                    size_t b_len_u32, uint32_t degree, uint64_t modulus, uint64_t *d_out);
int bc_fhe_poly_sub_check(size_t a_len_u32, size_t b_len_u32, uint32_t degree, uint64_t modulus);
int bc_fhe_poly_sub(bc_ctx *ctx, const uint64_t *d_a, size_t a_len_u32, const uint64_t *d_b,
                    size_t b_len_u32, uint32_t degree, uint64_t modulus, uint64_t *d_out);
int bc_fhe_poly_mul_check(size_t a_len_u32, size_t b_len_u32, uint32_t degree, uint64_t modulus);
int bc_fhe_poly_mul(bc_ctx *ctx, const uint64_t *d_a, size_t a_len_u32, const uint64_t *d_b,
                    size_t b_len_u32, uint32_t degree, uint64_t modulus, uint64_t *d_out);

/* fhe_rotate.rs:91-183 + fhe_rotate.wgsl.  Galois automorphism
 * X -> X^g, g = 2r + 1 with r = rotation (rotation + degree when negative):
 * coefficient i moves to p = i g mod 2N, and where p >= N it lands at p - N
 * as modulus - c (0 stays 0; 64-bit wrap-around for c > modulus, as the
 * shader computes it).  Bit-exact with the reference for any input.
 * Checks: degree a power of 2 >= 4, |rotation| <= degree / 2 (INT32_MIN is
 * rejected), input length; all BC_ERR_INVALID_INPUT.  d_out must not be
 * d_in. */
int bc_fhe_rotate_check(size_t input_len_u32, uint32_t degree, int32_t rotation, uint64_t modulus);
int bc_fhe_rotate(bc_ctx *ctx, const uint64_t *d_in, size_t input_len_u32, uint32_t degree,
                  int32_t rotation, uint64_t modulus, uint64_t *d_out);
/* Galois element 2r + 1 FheRotate uses for a rotation (0 when out of range). */
uint32_t bc_rotation_galois(uint32_t degree, int32_t rotation);

/* fhe_modulus_switch.rs:85-166 + .wgsl.  c' = round(c * new / old) mod new
 * (ties round up) per coefficient, exact for any u64 c.  The reference's
 * shader forms c * new in 64 bits; it matches this result whenever
 * c * new < 2^64 and old <= 2^63, and wraps otherwise.
 * Checks: degree, new < old, input length; all BC_ERR_INVALID_INPUT. */
int bc_fhe_modulus_switch_check(size_t input_len_u32, uint32_t degree, uint64_t modulus_old,
                                uint64_t modulus_new);
int bc_fhe_modulus_switch(bc_ctx *ctx, const uint64_t *d_in, size_t input_len_u32, uint32_t degree,
                          uint64_t modulus_old, uint64_t modulus_new, uint64_t *d_out);

/* fhe_key_switch.rs:101-222 + .wgsl.  Checks degree, 2 <= decomp_base <=
 * 2^24, 1 <= decomp_levels <= 32 and the input length (BC_ERR_INVALID_INPUT).
 * The result is a copy of the input: the reference's second pass
 * (accumulate_switched) stores its input buffer over the digits of the
 * first.  bc_decompose computes the digits themselves. */
int bc_fhe_key_switch_check(size_t input_len_u32, uint32_t degree, uint64_t modulus,
                            uint32_t decomp_base, uint32_t decomp_levels);
int bc_fhe_key_switch(bc_ctx *ctx, const uint64_t *d_in, size_t input_len_u32, uint32_t degree,
                      uint64_t modulus, uint32_t decomp_base, uint32_t decomp_levels,
                      uint64_t *d_out);

/* ------------------------------------------------ batched plans (new path)
 * A plan holds, for n_limbs RNS limbs of one degree N, the device twiddle
 * tables (with Shoup companions), N^-1 and the kernel choice.
 *
 * BC_NTT_CYCLIC: roots[i] is the N-th root omega_i and inv_roots[i] the root
 *   used by the inverse (NULL: the modular inverse of roots[i]).  Forward and
 *   inverse compute exactly the reference's DIT network, for any root value.
 * BC_NTT_NEGACYCLIC: roots[i] is a primitive 2N-th root psi_i (psi^N == -1
 *   mod q is checked); forward A_k = sum_j a_j psi^{j(2k+1)}, inverse its
 *   exact inverse, both in natural order.  inv_roots must be NULL.
 *
 * Moduli: q < 2^31 runs 32-bit Shoup arithmetic, 2^31 <= q < 2^62 runs
 * 64-bit Shoup/Harvey arithmetic; larger moduli are rejected. */
typedef enum bc_ntt_mode { BC_NTT_CYCLIC = 0, BC_NTT_NEGACYCLIC = 1 } bc_ntt_mode;

/* Element (limb l, polynomial p, coefficient j) of a batch lives at
 * base[l * limb_stride + p * poly_stride + j] (strides in u64 elements).
 * A NULL layout means limb-major contiguous: poly_stride = N,
 * limb_stride = batch * N. */
typedef struct bc_layout {
    int64_t limb_stride;
    int64_t poly_stride;
} bc_layout;

typedef struct bc_plan_info {
    uint32_t degree;
    uint32_t n_limbs;
    int32_t mode;
    int32_t word_bits;        /* 32 or 64: arithmetic width chosen from the moduli */
    int32_t kernel_kind;      /* 0 single-CTA shared memory, 1 cluster, 2 multi-pass */
    int32_t cluster_size;     /* CTAs per polynomial for kind 1 */
    uint64_t table_bytes;     /* device bytes of twiddle tables */
} bc_plan_info;

int bc_plan_create(bc_ctx *ctx, uint32_t degree, uint32_t n_limbs, const uint64_t *moduli,
                   const uint64_t *roots, const uint64_t *inv_roots, int mode,
                   bc_plan **out);
int bc_plan_destroy(bc_plan *plan);
int bc_plan_info_get(const bc_plan *plan, bc_plan_info *out);

/* Forward / inverse transform of `batch` polynomials per limb (all limbs).
 * In place (d_in == d_out) is allowed.  Asynchronous on `stream`
 * (NULL: the context stream).  The multi-pass path (kernel_kind 2, and
 * layouts the fast kernels cannot take above the shared-memory size) takes
 * a batch-sized temporary from the context's stream-ordered memory pool and
 * returns it on the same stream: calls on one plan from several streams or
 * threads never share it, and no call synchronizes. */
int bc_ntt_forward(bc_plan *plan, const uint64_t *d_in, uint64_t *d_out, uint32_t batch,
                   const bc_layout *layout, void *stream);
int bc_ntt_inverse(bc_plan *plan, const uint64_t *d_in, uint64_t *d_out, uint32_t batch,
                   const bc_layout *layout, void *stream);
/* Coefficient-wise C = A + B, A - B, A * B mod q_l over the whole batch,
 * with the semantics of bc_fhe_poly_add / _sub / _mul (inputs any u64). */
int bc_poly_add(bc_plan *plan, const uint64_t *d_a, const uint64_t *d_b, uint64_t *d_c,
                uint32_t batch, const bc_layout *layout, void *stream);
int bc_poly_sub(bc_plan *plan, const uint64_t *d_a, const uint64_t *d_b, uint64_t *d_c,
                uint32_t batch, const bc_layout *layout, void *stream);
int bc_poly_mul(bc_plan *plan, const uint64_t *d_a, const uint64_t *d_b, uint64_t *d_c,
                uint32_t batch, const bc_layout *layout, void *stream);
/* Transform fused with the pointwise product:
 *   bc_ntt_forward_mul: C = NTT(A) * B^, the product in the forward's epilogue;
 *   bc_ntt_inverse_mul: C = INTT(A^ * B^), the product in the inverse's prologue.
 * A^, B^ and the forward's result use bc_ntt_forward's natural order.  B^
 * words are reduced mod q_l first (a word >= 2^32 given to a plan whose moduli
 * are below 2^31 is reported as BC_ERR_INVALID_INPUT at the next
 * bc_ctx_sync, as for the transforms' inputs).  On BC_NTT_NEGACYCLIC plans
 * with the cluster kernels (16-byte aligned operands, even strides) this is
 * one launch moving 24N bytes per polynomial; other plans and layouts run a
 * transform launch and a pointwise launch, with the same result.  C may alias
 * A or B^. */
int bc_ntt_forward_mul(bc_plan *plan, const uint64_t *d_a, const uint64_t *d_b_hat, uint64_t *d_c,
                       uint32_t batch, const bc_layout *layout, void *stream);
int bc_ntt_inverse_mul(bc_plan *plan, const uint64_t *d_a_hat, const uint64_t *d_b_hat,
                       uint64_t *d_c, uint32_t batch, const bc_layout *layout, void *stream);
/* Transform fused with FhePolyAdd / FhePolySub (ops/fhe_poly_add.rs:67,
 * fhe_poly_sub.rs:47), the coefficient-wise steps on either side of it:
 *   bc_ntt_forward_add / _sub: C = NTT(A) +- B^ mod q, in the forward's epilogue;
 *   bc_ntt_inverse_add / _sub: C = INTT(A^ +- B^ mod q), in the inverse's prologue.
 * Exact mod q_l for any input words (A^ and B^ are reduced first; for inputs
 * below q that is the reference ops' result).  Layouts, aliasing, the
 * one-launch condition and the input-range report are those of
 * bc_ntt_forward_mul; otherwise a transform launch and a coefficient launch
 * give the same result. */
int bc_ntt_forward_add(bc_plan *plan, const uint64_t *d_a, const uint64_t *d_b_hat, uint64_t *d_c,
                       uint32_t batch, const bc_layout *layout, void *stream);
int bc_ntt_forward_sub(bc_plan *plan, const uint64_t *d_a, const uint64_t *d_b_hat, uint64_t *d_c,
                       uint32_t batch, const bc_layout *layout, void *stream);
int bc_ntt_inverse_add(bc_plan *plan, const uint64_t *d_a_hat, const uint64_t *d_b_hat,
                       uint64_t *d_c, uint32_t batch, const bc_layout *layout, void *stream);
int bc_ntt_inverse_sub(bc_plan *plan, const uint64_t *d_a_hat, const uint64_t *d_b_hat,
                       uint64_t *d_c, uint32_t batch, const bc_layout *layout, void *stream);
/* C = A * B mod q_l, coefficient-wise. */
int bc_pointwise_mul(bc_plan *plan, const uint64_t *d_a, const uint64_t *d_b, uint64_t *d_c,
                     uint32_t batch, const bc_layout *layout, void *stream);
/* C = INTT(NTT(A) * NTT(B)) per (limb, polynomial).  On the cluster kernels
 * (2^10 <= N <= 2^17, 16-byte aligned operands, even strides, not
 * A == B == C) negacyclic plans, and cyclic plans whose roots are all
 * primitive N-th roots of unity with inv_root = root^-1, run two launches:
 * NTT(B) into C, then one fused kernel C = INTT(NTT(A) * C) whose inverse is
 * a Gentleman-Sande network (for those roots it equals the reference's
 * FheFastPolyMul chain bit for bit).  Otherwise, up to N = 2^14 (moduli below
 * 2^31) or 2^13 (wider moduli), one fused shared-memory kernel.  Neither
 * allocates.  Every other case (N >= 2^18, cyclic plans with a non-primitive
 * root above the fused size, other layouts) transforms both operands into a
 * temporary, multiplies and runs the inverse into C, needing the default
 * layout (layout NULL or compact); the temporary comes from the context's
 * stream-ordered memory pool and is released on the same stream, so the call
 * does not synchronize. */
int bc_polymul(bc_plan *plan, const uint64_t *d_a, const uint64_t *d_b, uint64_t *d_c,
               uint32_t batch, const bc_layout *layout, void *stream);

/* Largest batch * n_limbs * N that bc_polymul_static_scratch accepts where
 * bc_polymul would allocate (2^21 coefficients per operand; the buffer is
 * 32 MiB). */
#define BC_POLYMUL_STATIC_MAX_COEFFS (1u << 21)

/* bc_polymul that never allocates device memory.  No counterpart in the
 * reference: FheFastPolyMul::execute (ops/fhe_fast_poly_mul.rs:122)
 * allocates its intermediates and output on every call.
 *
 * Who needs it: on its unfused path (see bc_polymul: N >= 2^18, cyclic plans
 * with a non-primitive root above the fused size, layouts the fused kernels
 * cannot take) bc_polymul takes a temporary from the context's memory pool
 * on every call, and the pool grows with fresh device memory when it holds
 * none free.  A caller cannot afford that when the device memory is already
 * reserved by another allocator (a framework's caching pool leaves the
 * driver nothing to hand out), or when it runs under a fixed device-memory
 * budget that steady-state serving must not grow.  This entry point keeps
 * the temporary in one fixed buffer per device in the library's static
 * device memory instead.  It computes the same result as bc_polymul and
 * neither allocates nor synchronizes.
 *
 * Limits: where bc_polymul would allocate, batch * n_limbs * N must not
 * exceed BC_POLYMUL_STATIC_MAX_COEFFS, and `layout` must be NULL or the
 * default compact layout.  Larger or strided calls fail with
 * BC_ERR_INVALID_INPUT / BC_ERR_UNSUPPORTED before any work is queued.
 * Where bc_polymul's fused kernels apply it is bc_polymul, with no limit.
 *
 * Sharing: every call on a GPU uses the same buffer.  Calls on one stream
 * are ordered and safe.  Calls that overlap in time race on the buffer and
 * give wrong results: other streams, other host threads, other plans or
 * contexts on the same GPU.  The caller must serialize them.
 *
 * Set-up: every call looks up the buffer's device address on the current
 * device (cudaGetSymbolAddress), so the address stays right after a device
 * reset; the first call on each device may make the driver load the
 * library's device code, so make that first call before any stream capture.
 * Nothing in the buffer needs to start at zero: every word is written
 * before it is read. */
int bc_polymul_static_scratch(bc_plan *plan, const uint64_t *d_a, const uint64_t *d_b,
                              uint64_t *d_c, uint32_t batch, const bc_layout *layout,
                              void *stream);

/* Galois automorphism X -> X^galois (galois odd, < 2N) of every polynomial
 * of the batch, with bc_fhe_rotate's semantics and limb l's modulus for the
 * negation.  d_in and d_out must not overlap. */
int bc_automorphism(bc_plan *plan, const uint64_t *d_in, uint64_t *d_out, uint32_t batch,
                    const bc_layout *layout, uint32_t galois, void *stream);
/* bc_fhe_modulus_switch's map over `count` words (any count; in place
 * allowed); asynchronous on `stream`.  Needs modulus_new < modulus_old. */
int bc_modulus_switch(bc_ctx *ctx, const uint64_t *d_in, uint64_t *d_out, size_t count,
                      uint64_t modulus_old, uint64_t modulus_new, void *stream);
/* Base-B digits of `count` words, the decomposition fhe_key_switch.wgsl:71-84
 * describes: d_out[l * count + i] = floor(d_in[i] / base^l) mod base for
 * l < levels (digit-major: each digit is a polynomial for the key-switching
 * product).  2 <= base <= 2^24, 1 <= levels <= 32; d_out holds
 * levels * count words and must not overlap d_in. */
int bc_decompose(bc_ctx *ctx, const uint64_t *d_in, uint64_t *d_out, size_t count, uint32_t base,
                 uint32_t levels, void *stream);

/* Seeded synthetic coefficients, uniform in [0, q_l): element (l, p, j) of
 * the batch gets value(seed, ((l * total_polys + first_poly + p) * N + j)),
 * value(s, g) = floor(splitmix64(s + (g + 1) * 0x9E3779B97F4A7C15) * q / 2^64). */
int bc_fill_uniform(bc_plan *plan, uint64_t *d_out, uint32_t batch, const bc_layout *layout,
                    uint64_t seed, uint64_t first_poly, uint64_t total_polys, void *stream);
/* Order-sensitive 64-bit digest of `count` u64 words for cross-GPU checks:
 * sum_i splitmix64(x_i ^ ((first_index + i) * 0xD1B54A32D192ED03)) mod 2^64,
 * written to *d_out.  With first_index = the global index of d_in[0], the
 * digests of the shards of an array add up (mod 2^64) to the digest of the
 * whole array, whatever the number of GPUs. */
int bc_digest(bc_ctx *ctx, const uint64_t *d_in, size_t count, uint64_t first_index,
              uint64_t *d_out, void *stream);

/* Integer-pipe peak of this GPU for the plans' butterfly arithmetic
 * (word_bits 32: q < 2^31 Shoup with lazy [0, 2q) reduction; 64: q < 2^62
 * Shoup/Harvey): register-only Cooley-Tukey butterflies on every SM, timed
 * with CUDA events on the context stream.  The NTT roofline is the slower
 * of 16N bytes at HBM bandwidth and (N/2) log2 N butterflies at this rate.
 * Takes a few milliseconds; synchronizes the context stream. */
int bc_calibrate_butterflies(bc_ctx *ctx, int word_bits, double *butterflies_per_s);

/* ------------------------------------------------------- multi-GPU split */
/* Contiguous balanced split of `units` over `shards`: shard s gets
 * [begin, begin + count) with sizes differing by at most one. */
int bc_partition(uint64_t units, uint32_t shards, uint32_t shard, uint64_t *begin,
                 uint64_t *count);

/* ------------------------------------------- host helpers (no GPU needed) */
/* i-th (0-based) largest prime q < 2^bits with q == 1 mod 2N (0 if none). */
uint64_t bc_ntt_prime(uint32_t bits, uint32_t degree, uint32_t index);
/* psi = g^((q-1)/2N), g the smallest generator of Z_q^* (q prime). */
uint64_t bc_negacyclic_root(uint64_t modulus, uint32_t degree);
/* Host copy of the device twiddle table entry k (1 <= k < N) of limb 0 of a
 * plan description, without a GPU: table 0 forward, 1 inverse.  Writes the
 * twiddle and its Shoup companion.  For tests of the table generator. */
int bc_debug_twiddle(uint32_t degree, uint64_t modulus, uint64_t root, uint64_t inv_root,
                     int mode, int table, uint32_t k, uint64_t *w, uint64_t *w_shoup);

#ifdef __cplusplus
}
#endif
#endif /* BARRACUDA_FHE_H */
