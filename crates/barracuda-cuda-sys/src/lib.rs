//! Bindings to `libbarracuda_fhe`, the B200-native (sm_100a) implementation of
//! barraCuda's FHE hot path: forward NTT, inverse INTT, the pointwise modular
//! product between them and the NTT-based polynomial product, over RNS limbs
//! and polynomial batches.
//!
//! barraCuda keeps `#![forbid(unsafe_code)]` in `crates/barracuda` and
//! `crates/barracuda-core`; every `unsafe` block of the CUDA backend lives in
//! this crate instead, the way `crates/barracuda-spirv` isolates its own FFI.
//! Two layers:
//!
//! - [`ffi`]: the C ABI of `include/barracuda_fhe.h`, declared one to one
//!   (same names, argument order and types).
//! - [`safe`]: owned handles ([`safe::Context`], [`safe::DeviceBuffer`],
//!   [`safe::Plan`]) and `Result`-returning calls that the FHE ops in
//!   `crates/barracuda` call from safe code.  Status codes map one to one onto
//!   `BarracudaError` variants ([`Status`]).
//!
//! Data layout: a polynomial of degree N is N little-endian `u64`
//! coefficients, byte-identical to the reference's `[lo32, hi32]` `u32`-pair
//! tensors (`Tensor::len() == 2N`).

#![deny(unsafe_op_in_unsafe_fn)]

/// The C ABI (`include/barracuda_fhe.h`), declared one to one.
#[allow(non_camel_case_types)]
pub mod ffi {
    use std::ffi::{c_char, c_int, c_void};

    /// `BC_ABI_VERSION`: bumped when a declaration below changes.
    pub const BC_ABI_VERSION: c_int = 1;

    pub const BC_OK: c_int = 0;
    pub const BC_ERR_DEVICE: c_int = 1;
    pub const BC_ERR_INVALID_INPUT: c_int = 2;
    pub const BC_ERR_OUT_OF_MEMORY: c_int = 3;
    pub const BC_ERR_DEVICE_LOST: c_int = 4;
    pub const BC_ERR_GPU: c_int = 5;
    pub const BC_ERR_UNSUPPORTED: c_int = 6;
    pub const BC_ERR_DEVICE_NOT_AVAILABLE: c_int = 7;
    pub const BC_ERR_EXECUTION: c_int = 8;
    pub const BC_ERR_INTERNAL: c_int = 9;

    /// `bc_ntt_mode`: the reference's cyclic transform, or the negacyclic
    /// (X^N + 1) transform with a 2N-th root psi.
    pub const BC_NTT_CYCLIC: c_int = 0;
    pub const BC_NTT_NEGACYCLIC: c_int = 1;

    /// `BC_POLYMUL_STATIC_MAX_COEFFS`: the limit of `bc_polymul_static_scratch`
    /// (batch * n_limbs * N per operand) where `bc_polymul` would allocate.
    pub const BC_POLYMUL_STATIC_MAX_COEFFS: u32 = 1 << 21;

    /// Opaque per-GPU context (stream, plan cache, device status word).
    #[repr(C)]
    pub struct bc_ctx {
        _private: [u8; 0],
    }

    /// Opaque batched transform plan (twiddle tables for n_limbs moduli).
    #[repr(C)]
    pub struct bc_plan {
        _private: [u8; 0],
    }

    /// Element (limb l, polynomial p, coefficient j) sits at
    /// `l * limb_stride + p * poly_stride + j` (in u64 words).
    #[repr(C)]
    #[derive(Clone, Copy, Debug, PartialEq, Eq)]
    pub struct bc_layout {
        pub limb_stride: i64,
        pub poly_stride: i64,
    }

    /// What a plan chose (`bc_plan_info_get`).
    #[repr(C)]
    #[derive(Clone, Copy, Debug, Default)]
    pub struct bc_plan_info {
        pub degree: u32,
        pub n_limbs: u32,
        pub mode: i32,
        pub word_bits: i32,
        pub kernel_kind: i32,
        pub cluster_size: i32,
        pub table_bytes: u64,
    }

    extern "C" {
        // ---- basics
        pub fn bc_last_error() -> *const c_char;
        pub fn bc_abi_version() -> c_int;
        pub fn bc_device_count(count: *mut c_int) -> c_int;
        pub fn bc_ctx_create(device: c_int, out: *mut *mut bc_ctx) -> c_int;
        pub fn bc_ctx_destroy(ctx: *mut bc_ctx) -> c_int;
        pub fn bc_ctx_device(ctx: *const bc_ctx, device: *mut c_int) -> c_int;
        pub fn bc_ctx_stream(ctx: *mut bc_ctx, stream: *mut *mut c_void) -> c_int;
        pub fn bc_ctx_sync(ctx: *mut bc_ctx) -> c_int;

        // ---- buffers
        pub fn bc_buf_alloc(ctx: *mut bc_ctx, bytes: usize, dptr: *mut *mut c_void) -> c_int;
        pub fn bc_buf_free(ctx: *mut bc_ctx, dptr: *mut c_void) -> c_int;
        pub fn bc_buf_h2d(ctx: *mut bc_ctx, dst: *mut c_void, src: *const c_void, bytes: usize) -> c_int;
        pub fn bc_buf_d2h(ctx: *mut bc_ctx, dst: *mut c_void, src: *const c_void, bytes: usize) -> c_int;
        pub fn bc_buf_h2d_async(
            ctx: *mut bc_ctx,
            dst: *mut c_void,
            src: *const c_void,
            bytes: usize,
            stream: *mut c_void,
        ) -> c_int;
        pub fn bc_buf_d2h_async(
            ctx: *mut bc_ctx,
            dst: *mut c_void,
            src: *const c_void,
            bytes: usize,
            stream: *mut c_void,
        ) -> c_int;
        pub fn bc_host_alloc(bytes: usize, hptr: *mut *mut c_void) -> c_int;
        pub fn bc_host_free(hptr: *mut c_void) -> c_int;

        // ---- reference op API (synchronous; lengths in u32 words)
        pub fn bc_compute_primitive_root(degree: u32, modulus: u64) -> u64;
        pub fn bc_compute_inverse_root(degree: u32, modulus: u64, root: u64) -> u64;
        pub fn bc_fhe_ntt_check(input_len_u32: usize, degree: u32, modulus: u64, root_of_unity: u64) -> c_int;
        pub fn bc_fhe_ntt(
            ctx: *mut bc_ctx,
            d_in: *const u64,
            input_len_u32: usize,
            degree: u32,
            modulus: u64,
            root_of_unity: u64,
            d_out: *mut u64,
        ) -> c_int;
        pub fn bc_fhe_intt_check(input_len_u32: usize, degree: u32, modulus: u64, inv_root_of_unity: u64) -> c_int;
        pub fn bc_fhe_intt(
            ctx: *mut bc_ctx,
            d_in: *const u64,
            input_len_u32: usize,
            degree: u32,
            modulus: u64,
            inv_root_of_unity: u64,
            d_out: *mut u64,
        ) -> c_int;
        pub fn bc_fhe_pointwise_mul_check(a_len_u32: usize, b_len_u32: usize, degree: u32, modulus: u64) -> c_int;
        pub fn bc_fhe_pointwise_mul(
            ctx: *mut bc_ctx,
            d_a: *const u64,
            a_len_u32: usize,
            d_b: *const u64,
            b_len_u32: usize,
            degree: u32,
            modulus: u64,
            d_out: *mut u64,
        ) -> c_int;
        pub fn bc_fhe_fast_poly_mul_check(
            a_len_u32: usize,
            b_len_u32: usize,
            degree: u32,
            modulus: u64,
            root_of_unity: u64,
        ) -> c_int;
        pub fn bc_fhe_fast_poly_mul(
            ctx: *mut bc_ctx,
            d_a: *const u64,
            a_len_u32: usize,
            d_b: *const u64,
            b_len_u32: usize,
            degree: u32,
            modulus: u64,
            root_of_unity: u64,
            d_out: *mut u64,
        ) -> c_int;
        pub fn bc_fhe_poly_add_check(a_len_u32: usize, b_len_u32: usize, degree: u32, modulus: u64) -> c_int;
        pub fn bc_fhe_poly_add(
            ctx: *mut bc_ctx,
            d_a: *const u64,
            a_len_u32: usize,
            d_b: *const u64,
            b_len_u32: usize,
            degree: u32,
            modulus: u64,
            d_out: *mut u64,
        ) -> c_int;
        pub fn bc_fhe_poly_sub_check(a_len_u32: usize, b_len_u32: usize, degree: u32, modulus: u64) -> c_int;
        pub fn bc_fhe_poly_sub(
            ctx: *mut bc_ctx,
            d_a: *const u64,
            a_len_u32: usize,
            d_b: *const u64,
            b_len_u32: usize,
            degree: u32,
            modulus: u64,
            d_out: *mut u64,
        ) -> c_int;
        pub fn bc_fhe_poly_mul_check(a_len_u32: usize, b_len_u32: usize, degree: u32, modulus: u64) -> c_int;
        pub fn bc_fhe_poly_mul(
            ctx: *mut bc_ctx,
            d_a: *const u64,
            a_len_u32: usize,
            d_b: *const u64,
            b_len_u32: usize,
            degree: u32,
            modulus: u64,
            d_out: *mut u64,
        ) -> c_int;
        pub fn bc_fhe_rotate_check(input_len_u32: usize, degree: u32, rotation: i32, modulus: u64) -> c_int;
        pub fn bc_fhe_rotate(
            ctx: *mut bc_ctx,
            d_in: *const u64,
            input_len_u32: usize,
            degree: u32,
            rotation: i32,
            modulus: u64,
            d_out: *mut u64,
        ) -> c_int;
        pub fn bc_rotation_galois(degree: u32, rotation: i32) -> u32;
        pub fn bc_fhe_modulus_switch_check(
            input_len_u32: usize,
            degree: u32,
            modulus_old: u64,
            modulus_new: u64,
        ) -> c_int;
        pub fn bc_fhe_modulus_switch(
            ctx: *mut bc_ctx,
            d_in: *const u64,
            input_len_u32: usize,
            degree: u32,
            modulus_old: u64,
            modulus_new: u64,
            d_out: *mut u64,
        ) -> c_int;
        pub fn bc_fhe_key_switch_check(
            input_len_u32: usize,
            degree: u32,
            modulus: u64,
            decomp_base: u32,
            decomp_levels: u32,
        ) -> c_int;
        pub fn bc_fhe_key_switch(
            ctx: *mut bc_ctx,
            d_in: *const u64,
            input_len_u32: usize,
            degree: u32,
            modulus: u64,
            decomp_base: u32,
            decomp_levels: u32,
            d_out: *mut u64,
        ) -> c_int;

        // ---- batched plans (asynchronous on `stream`; NULL = context stream)
        pub fn bc_plan_create(
            ctx: *mut bc_ctx,
            degree: u32,
            n_limbs: u32,
            moduli: *const u64,
            roots: *const u64,
            inv_roots: *const u64,
            mode: c_int,
            out: *mut *mut bc_plan,
        ) -> c_int;
        pub fn bc_plan_destroy(plan: *mut bc_plan) -> c_int;
        pub fn bc_plan_info_get(plan: *const bc_plan, out: *mut bc_plan_info) -> c_int;
        pub fn bc_ntt_forward(
            plan: *mut bc_plan,
            d_in: *const u64,
            d_out: *mut u64,
            batch: u32,
            layout: *const bc_layout,
            stream: *mut c_void,
        ) -> c_int;
        pub fn bc_ntt_inverse(
            plan: *mut bc_plan,
            d_in: *const u64,
            d_out: *mut u64,
            batch: u32,
            layout: *const bc_layout,
            stream: *mut c_void,
        ) -> c_int;
        pub fn bc_poly_add(
            plan: *mut bc_plan,
            d_a: *const u64,
            d_b: *const u64,
            d_c: *mut u64,
            batch: u32,
            layout: *const bc_layout,
            stream: *mut c_void,
        ) -> c_int;
        pub fn bc_poly_sub(
            plan: *mut bc_plan,
            d_a: *const u64,
            d_b: *const u64,
            d_c: *mut u64,
            batch: u32,
            layout: *const bc_layout,
            stream: *mut c_void,
        ) -> c_int;
        pub fn bc_poly_mul(
            plan: *mut bc_plan,
            d_a: *const u64,
            d_b: *const u64,
            d_c: *mut u64,
            batch: u32,
            layout: *const bc_layout,
            stream: *mut c_void,
        ) -> c_int;
        pub fn bc_ntt_forward_mul(
            plan: *mut bc_plan,
            d_a: *const u64,
            d_b_hat: *const u64,
            d_c: *mut u64,
            batch: u32,
            layout: *const bc_layout,
            stream: *mut c_void,
        ) -> c_int;
        pub fn bc_ntt_inverse_mul(
            plan: *mut bc_plan,
            d_a_hat: *const u64,
            d_b_hat: *const u64,
            d_c: *mut u64,
            batch: u32,
            layout: *const bc_layout,
            stream: *mut c_void,
        ) -> c_int;
        pub fn bc_ntt_forward_add(
            plan: *mut bc_plan,
            d_a: *const u64,
            d_b_hat: *const u64,
            d_c: *mut u64,
            batch: u32,
            layout: *const bc_layout,
            stream: *mut c_void,
        ) -> c_int;
        pub fn bc_ntt_forward_sub(
            plan: *mut bc_plan,
            d_a: *const u64,
            d_b_hat: *const u64,
            d_c: *mut u64,
            batch: u32,
            layout: *const bc_layout,
            stream: *mut c_void,
        ) -> c_int;
        pub fn bc_ntt_inverse_add(
            plan: *mut bc_plan,
            d_a_hat: *const u64,
            d_b_hat: *const u64,
            d_c: *mut u64,
            batch: u32,
            layout: *const bc_layout,
            stream: *mut c_void,
        ) -> c_int;
        pub fn bc_ntt_inverse_sub(
            plan: *mut bc_plan,
            d_a_hat: *const u64,
            d_b_hat: *const u64,
            d_c: *mut u64,
            batch: u32,
            layout: *const bc_layout,
            stream: *mut c_void,
        ) -> c_int;
        pub fn bc_pointwise_mul(
            plan: *mut bc_plan,
            d_a: *const u64,
            d_b: *const u64,
            d_c: *mut u64,
            batch: u32,
            layout: *const bc_layout,
            stream: *mut c_void,
        ) -> c_int;
        pub fn bc_polymul(
            plan: *mut bc_plan,
            d_a: *const u64,
            d_b: *const u64,
            d_c: *mut u64,
            batch: u32,
            layout: *const bc_layout,
            stream: *mut c_void,
        ) -> c_int;
        pub fn bc_polymul_static_scratch(
            plan: *mut bc_plan,
            d_a: *const u64,
            d_b: *const u64,
            d_c: *mut u64,
            batch: u32,
            layout: *const bc_layout,
            stream: *mut c_void,
        ) -> c_int;
        pub fn bc_automorphism(
            plan: *mut bc_plan,
            d_in: *const u64,
            d_out: *mut u64,
            batch: u32,
            layout: *const bc_layout,
            galois: u32,
            stream: *mut c_void,
        ) -> c_int;
        pub fn bc_modulus_switch(
            ctx: *mut bc_ctx,
            d_in: *const u64,
            d_out: *mut u64,
            count: usize,
            modulus_old: u64,
            modulus_new: u64,
            stream: *mut c_void,
        ) -> c_int;
        pub fn bc_decompose(
            ctx: *mut bc_ctx,
            d_in: *const u64,
            d_out: *mut u64,
            count: usize,
            base: u32,
            levels: u32,
            stream: *mut c_void,
        ) -> c_int;

        // ---- inputs, verification, calibration, sharding
        pub fn bc_fill_uniform(
            plan: *mut bc_plan,
            d_out: *mut u64,
            batch: u32,
            layout: *const bc_layout,
            seed: u64,
            first_poly: u64,
            total_polys: u64,
            stream: *mut c_void,
        ) -> c_int;
        pub fn bc_digest(
            ctx: *mut bc_ctx,
            d_in: *const u64,
            count: usize,
            first_index: u64,
            d_out: *mut u64,
            stream: *mut c_void,
        ) -> c_int;
        pub fn bc_calibrate_butterflies(ctx: *mut bc_ctx, word_bits: c_int, butterflies_per_s: *mut f64) -> c_int;
        pub fn bc_partition(units: u64, shards: u32, shard: u32, begin: *mut u64, count: *mut u64) -> c_int;
        pub fn bc_ntt_prime(bits: u32, degree: u32, index: u32) -> u64;
        pub fn bc_negacyclic_root(modulus: u64, degree: u32) -> u64;
        pub fn bc_debug_twiddle(
            degree: u32,
            modulus: u64,
            root: u64,
            inv_root: u64,
            mode: c_int,
            table: c_int,
            k: u32,
            w: *mut u64,
            w_shoup: *mut u64,
        ) -> c_int;
    }
}

use std::ffi::{c_int, CStr};
use std::fmt;

/// A failed call: the status code and the library's message for it.
///
/// The codes map one to one onto `BarracudaError` (crates/barracuda/src/error.rs):
/// 1 `Device` (op validation, same text as the Rust constructors),
/// 2 `InvalidInput`, 3 `OutOfMemory`, 4 `DeviceLost`, 5 `Gpu`,
/// 6 `UnsupportedOperation`, 7 `DeviceNotAvailable`, 8 `ExecutionError`,
/// 9 `Internal`.
#[derive(Clone, Debug, PartialEq, Eq)]
pub struct Status {
    pub code: i32,
    pub message: String,
}

impl fmt::Display for Status {
    fn fmt(&self, f: &mut fmt::Formatter<'_>) -> fmt::Result {
        write!(f, "barracuda_fhe status {}: {}", self.code, self.message)
    }
}

impl std::error::Error for Status {}

/// Converts a status code into a `Result`, copying the per-thread message.
pub fn check(code: c_int) -> Result<(), Status> {
    if code == ffi::BC_OK {
        return Ok(());
    }
    // SAFETY: bc_last_error returns a NUL-terminated string owned by the
    // library's per-thread buffer; it is copied before any other call.
    let message = unsafe { CStr::from_ptr(ffi::bc_last_error()) }.to_string_lossy().into_owned();
    Err(Status { code, message })
}

/// Owned handles and safe calls for `crates/barracuda` (which forbids unsafe).
pub mod safe {
    use super::{check, ffi, Status};
    use std::ffi::{c_int, c_void};
    use std::ptr::{self, NonNull};
    use std::sync::Arc;

    /// One GPU: a non-blocking stream, a plan cache and the status word.
    /// Created where the reference creates its `WgpuDevice`.
    pub struct Context {
        raw: NonNull<ffi::bc_ctx>,
    }

    // SAFETY: the library serialises use of a context's plan cache with a
    // mutex and orders launches on its stream; handles may cross threads.
    unsafe impl Send for Context {}
    unsafe impl Sync for Context {}

    impl Context {
        pub fn new(device: i32) -> Result<Arc<Context>, Status> {
            let mut raw = ptr::null_mut();
            // SAFETY: `raw` is a valid out-pointer.
            check(unsafe { ffi::bc_ctx_create(device, &mut raw) })?;
            let raw = NonNull::new(raw).ok_or_else(|| Status { code: ffi::BC_ERR_INTERNAL, message: "null context".into() })?;
            Ok(Arc::new(Context { raw }))
        }

        fn ptr(&self) -> *mut ffi::bc_ctx {
            self.raw.as_ptr()
        }

        /// Waits for the context stream and reports statuses kernels raised
        /// (a coefficient >= 2^32 on a plan whose moduli are below 2^31).
        pub fn sync(&self) -> Result<(), Status> {
            // SAFETY: the context is alive for &self.
            check(unsafe { ffi::bc_ctx_sync(self.ptr()) })
        }

        /// Device buffer of `words` u64 coefficients.
        pub fn alloc(self: &Arc<Self>, words: usize) -> Result<DeviceBuffer, Status> {
            let mut dptr = ptr::null_mut();
            // SAFETY: valid context and out-pointer.
            check(unsafe { ffi::bc_buf_alloc(self.ptr(), words * 8, &mut dptr) })?;
            Ok(DeviceBuffer { ctx: Arc::clone(self), ptr: dptr.cast(), words })
        }

        /// `create_fhe_poly_tensor` + `Tensor::from_data_pod`: uploads u64 words.
        pub fn upload(self: &Arc<Self>, data: &[u64]) -> Result<DeviceBuffer, Status> {
            let buf = self.alloc(data.len())?;
            // SAFETY: `buf` holds data.len() words; the source slice is valid.
            check(unsafe {
                ffi::bc_buf_h2d(self.ptr(), buf.ptr.cast(), data.as_ptr().cast(), data.len() * 8)
            })?;
            Ok(buf)
        }

        /// `FheNtt::new` + `execute`: `out` = NTT(`input`), cyclic, natural order.
        pub fn fhe_ntt(&self, input: &DeviceBuffer, degree: u32, modulus: u64, root: u64,
                       out: &mut DeviceBuffer) -> Result<(), Status> {
            out.expect(degree as usize)?;
            // SAFETY: both buffers are alive; the library checks the length
            // (in u32 words) against the degree before reading.
            check(unsafe {
                ffi::bc_fhe_ntt(self.ptr(), input.ptr, input.words * 2, degree, modulus, root, out.ptr)
            })
        }

        /// `FheIntt::new` + `execute`.
        pub fn fhe_intt(&self, input: &DeviceBuffer, degree: u32, modulus: u64, inv_root: u64,
                        out: &mut DeviceBuffer) -> Result<(), Status> {
            out.expect(degree as usize)?;
            // SAFETY: as in fhe_ntt.
            check(unsafe {
                ffi::bc_fhe_intt(self.ptr(), input.ptr, input.words * 2, degree, modulus, inv_root, out.ptr)
            })
        }

        /// `FhePointwiseMul::new` + `execute`.
        pub fn fhe_pointwise_mul(&self, a: &DeviceBuffer, b: &DeviceBuffer, degree: u32, modulus: u64,
                                 out: &mut DeviceBuffer) -> Result<(), Status> {
            out.expect(degree as usize)?;
            // SAFETY: as in fhe_ntt.
            check(unsafe {
                ffi::bc_fhe_pointwise_mul(self.ptr(), a.ptr, a.words * 2, b.ptr, b.words * 2, degree, modulus, out.ptr)
            })
        }

        /// `FheFastPolyMul::new` + `execute`: cyclic a * b mod (X^N - 1, q).
        pub fn fhe_fast_poly_mul(&self, a: &DeviceBuffer, b: &DeviceBuffer, degree: u32, modulus: u64,
                                 root: u64, out: &mut DeviceBuffer) -> Result<(), Status> {
            out.expect(degree as usize)?;
            // SAFETY: as in fhe_ntt.
            check(unsafe {
                ffi::bc_fhe_fast_poly_mul(self.ptr(), a.ptr, a.words * 2, b.ptr, b.words * 2, degree, modulus,
                                          root, out.ptr)
            })
        }
    }

    impl Drop for Context {
        fn drop(&mut self) {
            // SAFETY: the context was created by bc_ctx_create and is dropped once.
            unsafe {
                ffi::bc_ctx_destroy(self.ptr());
            }
        }
    }

    /// Caller-owned device memory of `words` u64 coefficients.
    pub struct DeviceBuffer {
        ctx: Arc<Context>,
        ptr: *mut u64,
        words: usize,
    }

    // SAFETY: a device pointer is not tied to a host thread.
    unsafe impl Send for DeviceBuffer {}
    unsafe impl Sync for DeviceBuffer {}

    impl DeviceBuffer {
        /// Number of u64 coefficients.
        pub fn words(&self) -> usize {
            self.words
        }

        /// `Tensor::len()`: the length in u32 words.
        pub fn len_u32(&self) -> usize {
            self.words * 2
        }

        fn expect(&self, words: usize) -> Result<(), Status> {
            if self.words < words {
                return Err(Status {
                    code: ffi::BC_ERR_INVALID_INPUT,
                    message: format!("output buffer holds {} words, {} needed", self.words, words),
                });
            }
            Ok(())
        }

        /// `Tensor::to_vec_u32` as u64 words.
        pub fn download(&self) -> Result<Vec<u64>, Status> {
            let mut out = vec![0u64; self.words];
            // SAFETY: `out` has room for the buffer's bytes.
            check(unsafe {
                ffi::bc_buf_d2h(self.ctx.ptr(), out.as_mut_ptr().cast(), self.ptr.cast::<c_void>(), self.words * 8)
            })?;
            Ok(out)
        }
    }

    impl Drop for DeviceBuffer {
        fn drop(&mut self) {
            // SAFETY: allocated by bc_buf_alloc on this context, freed once.
            unsafe {
                ffi::bc_buf_free(self.ctx.ptr(), self.ptr.cast());
            }
        }
    }

    /// Transform mode of a batched plan.
    #[derive(Clone, Copy, Debug, PartialEq, Eq)]
    pub enum Mode {
        /// The reference's cyclic transform with an N-th root omega.
        Cyclic,
        /// The negacyclic transform with a 2N-th root psi.
        Negacyclic,
    }

    /// Twiddle tables for `n_limbs` moduli of one degree; immutable after
    /// creation and shared by threads and streams.
    pub struct Plan {
        ctx: Arc<Context>,
        raw: NonNull<ffi::bc_plan>,
    }

    // SAFETY: a plan is immutable after creation (the library's contract).
    unsafe impl Send for Plan {}
    unsafe impl Sync for Plan {}

    impl Plan {
        pub fn new(ctx: &Arc<Context>, degree: u32, moduli: &[u64], roots: &[u64], mode: Mode)
                   -> Result<Plan, Status> {
            if moduli.len() != roots.len() {
                return Err(Status { code: ffi::BC_ERR_INVALID_INPUT, message: "one root per modulus".into() });
            }
            let mut raw = ptr::null_mut();
            let m: c_int = match mode {
                Mode::Cyclic => ffi::BC_NTT_CYCLIC,
                Mode::Negacyclic => ffi::BC_NTT_NEGACYCLIC,
            };
            // SAFETY: the slices hold n_limbs entries; inv_roots NULL lets the
            // plan derive them.
            check(unsafe {
                ffi::bc_plan_create(ctx.ptr(), degree, moduli.len() as u32, moduli.as_ptr(), roots.as_ptr(),
                                    ptr::null(), m, &mut raw)
            })?;
            let raw = NonNull::new(raw).ok_or_else(|| Status { code: ffi::BC_ERR_INTERNAL, message: "null plan".into() })?;
            Ok(Plan { ctx: Arc::clone(ctx), raw })
        }

        pub fn info(&self) -> Result<ffi::bc_plan_info, Status> {
            let mut info = ffi::bc_plan_info::default();
            // SAFETY: valid plan and out-pointer.
            check(unsafe { ffi::bc_plan_info_get(self.raw.as_ptr(), &mut info) })?;
            Ok(info)
        }

        fn layout_ptr(layout: Option<&ffi::bc_layout>) -> *const ffi::bc_layout {
            layout.map_or(ptr::null(), |l| l as *const _)
        }

        fn need(&self, buf: &DeviceBuffer, batch: u32, layout: Option<&ffi::bc_layout>) -> Result<(), Status> {
            let info = self.info()?;
            let n = info.degree as i64;
            let (ls, ps) = match layout {
                Some(l) => (l.limb_stride, l.poly_stride),
                None => (batch as i64 * n, n),
            };
            let last = (info.n_limbs as i64 - 1) * ls + (batch as i64 - 1) * ps + n;
            if batch == 0 || last > buf.words as i64 {
                return Err(Status {
                    code: ffi::BC_ERR_INVALID_INPUT,
                    message: format!("buffer of {} words is smaller than the layout needs ({last})", buf.words),
                });
            }
            Ok(())
        }

        /// Forward transform of every (limb, polynomial); queued on the context stream.
        pub fn forward(&self, input: &DeviceBuffer, out: &mut DeviceBuffer, batch: u32,
                       layout: Option<&ffi::bc_layout>) -> Result<(), Status> {
            self.need(input, batch, layout)?;
            self.need(out, batch, layout)?;
            // SAFETY: both buffers cover the layout (checked above).
            check(unsafe {
                ffi::bc_ntt_forward(self.raw.as_ptr(), input.ptr, out.ptr, batch, Self::layout_ptr(layout),
                                    ptr::null_mut())
            })
        }

        /// Inverse transform (N^-1 folded in).
        pub fn inverse(&self, input: &DeviceBuffer, out: &mut DeviceBuffer, batch: u32,
                       layout: Option<&ffi::bc_layout>) -> Result<(), Status> {
            self.need(input, batch, layout)?;
            self.need(out, batch, layout)?;
            // SAFETY: as in forward.
            check(unsafe {
                ffi::bc_ntt_inverse(self.raw.as_ptr(), input.ptr, out.ptr, batch, Self::layout_ptr(layout),
                                    ptr::null_mut())
            })
        }

        /// C = INTT(NTT(A) * NTT(B)).
        pub fn polymul(&self, a: &DeviceBuffer, b: &DeviceBuffer, c: &mut DeviceBuffer, batch: u32,
                       layout: Option<&ffi::bc_layout>) -> Result<(), Status> {
            self.need(a, batch, layout)?;
            self.need(b, batch, layout)?;
            self.need(c, batch, layout)?;
            // SAFETY: all three buffers cover the layout (checked above).
            check(unsafe {
                ffi::bc_polymul(self.raw.as_ptr(), a.ptr, b.ptr, c.ptr, batch, Self::layout_ptr(layout),
                                ptr::null_mut())
            })
        }

        /// Waits for the plan's context and reports kernel statuses.
        pub fn sync(&self) -> Result<(), Status> {
            self.ctx.sync()
        }
    }

    impl Drop for Plan {
        fn drop(&mut self) {
            // SAFETY: created by bc_plan_create, destroyed once; the library
            // waits for the context stream first.
            unsafe {
                ffi::bc_plan_destroy(self.raw.as_ptr());
            }
        }
    }

    /// The validation of each reference constructor, without running it
    /// (`FheNtt::new` and friends keep their signatures and messages).
    pub fn fhe_ntt_check(input_len_u32: usize, degree: u32, modulus: u64, root: u64) -> Result<(), Status> {
        // SAFETY: pure validation, no pointers.
        check(unsafe { ffi::bc_fhe_ntt_check(input_len_u32, degree, modulus, root) })
    }

    pub fn fhe_intt_check(input_len_u32: usize, degree: u32, modulus: u64, inv_root: u64) -> Result<(), Status> {
        // SAFETY: pure validation.
        check(unsafe { ffi::bc_fhe_intt_check(input_len_u32, degree, modulus, inv_root) })
    }

    pub fn fhe_pointwise_mul_check(a_len_u32: usize, b_len_u32: usize, degree: u32, modulus: u64)
                                   -> Result<(), Status> {
        // SAFETY: pure validation.
        check(unsafe { ffi::bc_fhe_pointwise_mul_check(a_len_u32, b_len_u32, degree, modulus) })
    }

    pub fn fhe_fast_poly_mul_check(a_len_u32: usize, b_len_u32: usize, degree: u32, modulus: u64, root: u64)
                                   -> Result<(), Status> {
        // SAFETY: pure validation.
        check(unsafe { ffi::bc_fhe_fast_poly_mul_check(a_len_u32, b_len_u32, degree, modulus, root) })
    }

    /// `compute_primitive_root` (fhe_ntt/mod.rs:210): same candidates and fallbacks.
    pub fn compute_primitive_root(degree: u32, modulus: u64) -> u64 {
        // SAFETY: pure function.
        unsafe { ffi::bc_compute_primitive_root(degree, modulus) }
    }

    /// `compute_inverse_root` (fhe_intt/mod.rs:202): 0 when not invertible.
    pub fn compute_inverse_root(degree: u32, modulus: u64, root: u64) -> u64 {
        // SAFETY: pure function.
        unsafe { ffi::bc_compute_inverse_root(degree, modulus, root) }
    }

    /// Balanced contiguous split of `units` over `shards`: (begin, count) of `shard`.
    pub fn partition(units: u64, shards: u32, shard: u32) -> Result<(u64, u64), Status> {
        let (mut begin, mut count) = (0u64, 0u64);
        // SAFETY: valid out-pointers.
        check(unsafe { ffi::bc_partition(units, shards, shard, &mut begin, &mut count) })?;
        Ok((begin, count))
    }
}

#[cfg(test)]
mod tests {
    use super::*;

    #[test]
    fn abi_version_matches() {
        // SAFETY: no arguments.
        assert_eq!(unsafe { ffi::bc_abi_version() }, ffi::BC_ABI_VERSION);
    }

    #[test]
    fn primitive_root_known_answer() {
        // g = 2 gives 2^4 = 16 with 16^2 = 1 (rejected); g = 3 gives 13
        assert_eq!(safe::compute_primitive_root(4, 17), 13);
    }

    #[test]
    fn validation_messages_match_the_reference() {
        // fhe_ntt/mod.rs:97-105: the length check comes first
        let e = safe::fhe_ntt_check(8, 3, 17, 4).unwrap_err();
        assert_eq!(e.code, ffi::BC_ERR_DEVICE);
        assert_eq!(e.message, "Input length 8 doesn't match expected 6 (degree 3 * 2)");
        let e = safe::fhe_ntt_check(6, 3, 17, 4).unwrap_err();
        assert!(e.message.contains("power of 2"), "{}", e.message);
    }
}
