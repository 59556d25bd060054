// bc_runtime.cpp -- contexts, device buffers, plans (twiddle tables), the
// batched transform entry points and the multi-GPU split of the C ABI.
#include "bc_runtime.hpp"

#include <algorithm>
#include <chrono>
#include <cstring>
#include <thread>

namespace bc {
const char *last_error_cstr();

int cuda_fail(cudaError_t e, const char *what) {
    int st = BC_ERR_GPU;
    switch (e) {
    case cudaErrorMemoryAllocation: st = BC_ERR_OUT_OF_MEMORY; break;
    case cudaErrorNoDevice:
    case cudaErrorInvalidDevice:
    case cudaErrorInsufficientDriver: st = BC_ERR_DEVICE_NOT_AVAILABLE; break;
    case cudaErrorIllegalAddress:
    case cudaErrorLaunchFailure:
    case cudaErrorIllegalInstruction:
    case cudaErrorMisalignedAddress:
    case cudaErrorHardwareStackError:
    case cudaErrorECCUncorrectable:
    case cudaErrorDevicesUnavailable: st = BC_ERR_DEVICE_LOST; break;
    default: break;
    }
    return fail(st, format("%s: %s", what, cudaGetErrorString(e)));
}

int use_device(const bc_ctx *ctx) {
    const cudaError_t e = cudaSetDevice(ctx->device);
    return e == cudaSuccess ? BC_OK : cuda_fail(e, "cudaSetDevice");
}

// Waits for `s`: polls for a short while first (a single reference-op call
// finishes within microseconds, and a blocking wait adds the thread's wake-up
// latency on top), then blocks.
cudaError_t wait_stream(cudaStream_t s) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t q = cudaStreamQuery(s);
        if (q != cudaErrorNotReady) return q;
        if (std::chrono::steady_clock::now() - t0 > std::chrono::microseconds(200)) break;
    }
    return cudaStreamSynchronize(s);
}

int ctx_sync(bc_ctx *ctx) {
    // kernels store into the mapped status word; once the stream is done its
    // value is visible on the host without a copy
    const cudaError_t e = wait_stream(ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "stream synchronize");
    volatile uint32_t *hs = ctx->h_status;
    const uint32_t st = *hs;
    if (st) {
        *hs = 0;
        if (st & kStatusInputRange)
            return fail(BC_ERR_INVALID_INPUT,
                        "coefficient >= 2^32 given to a transform whose moduli are below 2^31 "
                        "(inputs must be reduced; the reference is exact only below 2^32)");
        if (st & kStatusWaitTimeout)
            return fail(BC_ERR_EXECUTION, "a kernel gave up waiting for an asynchronous copy (results undefined)");
        return fail(BC_ERR_EXECUTION, format("kernel reported status 0x%x", st));
    }
    return BC_OK;
}

// ---------------------------------------------------------------- tables

namespace {

Word choose_word(const std::vector<uint64_t> &moduli) {
    uint64_t mx = 0;
    for (uint64_t q : moduli) mx = std::max(mx, q);
    if (mx < (1ull << 30)) return Word::W32Lazy4;
    if (mx < (1ull << 31)) return Word::W32Lazy2;
    return Word::W64;
}

bool is32(Word w) { return w != Word::W64; }

// Powers base^0 .. base^(count-1) mod q by repeated multiplication (the
// same sequence as compute_twiddle_factors, fhe_ntt/mod.rs:174-184).
std::vector<uint64_t> powers(uint64_t base, uint64_t q, uint32_t count) {
    std::vector<uint64_t> out(count);
    uint64_t p = 1 % q;
    for (uint32_t k = 0; k < count; ++k) {
        out[k] = p;
        p = mulmod(p, base, q);
    }
    return out;
}

uint32_t floor_log2(uint32_t k) {
    uint32_t l = 0;
    while ((k >> (l + 1)) != 0) ++l;
    return l;
}

// Twiddle value (no Shoup companion) of entry k in [1, N) of one table.
struct TableGen {
    uint32_t L = 0, N = 0;
    int mode = BC_NTT_CYCLIC;
    bool inverse = false;
    uint64_t q = 0, ninv = 0;
    std::vector<uint64_t> pw;  // powers of the table's base root

    bool gs_fold = false;  // cyclic inverse: N^-1 on the first entry (a GS network's last stage)

    void init(uint32_t logn, int md, bool inv, uint64_t modulus, uint64_t root, uint64_t inv_root,
              uint64_t n_inverse, bool fold_first = false) {
        L = logn;
        N = 1u << logn;
        mode = md;
        inverse = inv;
        gs_fold = fold_first;
        q = modulus;
        ninv = n_inverse;
        if (mode == BC_NTT_CYCLIC) {
            // CT-ordered DIT network: entry m + i (m = 2^s) is
            // r^(bitrev_s(i) * N / (2m)); exponents < N/2.
            pw = powers((inverse ? inv_root : root) % q, q, std::max(N / 2, 1u));
        } else {
            // negacyclic: psi^(+-bitrev_L(k)); exponents < N.
            pw = powers((inverse ? inv_root : root) % q, q, N);
        }
    }

    uint64_t value(uint32_t k) const {
        if (k == 0 || k >= N) return 0;
        uint64_t w;
        if (mode == BC_NTT_CYCLIC) {
            const uint32_t s = floor_log2(k);
            const uint32_t m = 1u << s, i = k - m;
            w = pw[static_cast<size_t>(s ? bitrev(i, s) : 0) * (N / (2 * m))];
            // last CT stage of the inverse (m = N/2) carries N^-1, or, for
            // the Gentleman-Sande form of the inverse, its last stage (k = 1)
            if (inverse && (gs_fold ? k == 1 : m == N / 2)) w = mulmod(w, ninv, q);
        } else {
            w = pw[bitrev(k, L)];
            // last GS stage (m = 1) carries N^-1
            if (inverse && k == 1) w = mulmod(w, ninv, q);
        }
        return w % q;
    }
};

}  // namespace

// Whether every limb's root of a cyclic plan is a primitive N-th root of
// unity whose stored inverse is its exact inverse (and N is invertible):
// then every radix-2 factorisation of the DFT agrees, and a Gentleman-Sande
// inverse equals the reference's Cooley-Tukey INTT bit for bit.  For any
// other root the reference's outputs depend on its exact stage structure
// (fhe_ntt.wgsl:223-241), which only the plan's own CT tables reproduce.
bool cyclic_roots_primitive(const bc_plan &p) {
    if (p.mode != BC_NTT_CYCLIC || p.degree < 2) return false;
    for (uint32_t l = 0; l < p.n_limbs; ++l) {
        const uint64_t q = p.moduli[l], w = p.roots[l] % q;
        if (q < 3 || q % 2 == 0 || p.limbs[l].ninv == 0) return false;
        if (powmod(w, p.degree, q) != 1 || powmod(w, p.degree / 2, q) != q - 1) return false;
        if (mulmod(w, p.inv_roots[l] % q, q) != 1) return false;
    }
    return true;
}

int plan_build_host(bc_plan &p, uint32_t degree, uint32_t n_limbs, const uint64_t *moduli,
                    const uint64_t *roots, const uint64_t *inv_roots, int mode,
                    std::vector<unsigned char> *fwd, std::vector<unsigned char> *inv) {
    if (degree == 0 || !is_pow2(degree))
        return fail(BC_ERR_INVALID_INPUT, format("degree %u must be a power of two", degree));
    if (n_limbs == 0) return fail(BC_ERR_INVALID_INPUT, "n_limbs must be at least 1");
    if (!moduli || !roots) return fail(BC_ERR_INVALID_INPUT, "moduli and roots must not be NULL");
    if (mode != BC_NTT_CYCLIC && mode != BC_NTT_NEGACYCLIC)
        return fail(BC_ERR_INVALID_INPUT, format("unknown transform mode %d", mode));
    if (mode == BC_NTT_NEGACYCLIC && inv_roots)
        return fail(BC_ERR_INVALID_INPUT, "negacyclic plans derive the inverse root; pass NULL");
    if (degree > (1u << 24))
        return fail(BC_ERR_UNSUPPORTED, format("degree %u above 2^24 is not supported", degree));
    p.degree = degree;
    p.logn = ilog2(degree);
    p.n_limbs = n_limbs;
    p.mode = mode;
    p.moduli.assign(moduli, moduli + n_limbs);
    p.roots.assign(roots, roots + n_limbs);
    p.inv_roots.resize(n_limbs);
    for (uint32_t l = 0; l < n_limbs; ++l) {
        const uint64_t q = moduli[l];
        if (q == 0) return fail(BC_ERR_INVALID_INPUT, format("modulus of limb %u is zero", l));
        if (q >= (1ull << 62))
            return fail(BC_ERR_UNSUPPORTED,
                        format("modulus %llu of limb %u is >= 2^62 (largest supported width)",
                               static_cast<unsigned long long>(q), l));
        if (mode == BC_NTT_NEGACYCLIC) {
            if (q < 3 || (q - 1) % (2ull * degree) != 0)
                return fail(BC_ERR_INVALID_INPUT,
                            format("modulus %llu of limb %u must satisfy q == 1 (mod 2N), N=%u",
                                   static_cast<unsigned long long>(q), l, degree));
            if (powmod(roots[l] % q, degree, q) != q - 1)
                return fail(BC_ERR_INVALID_INPUT,
                            format("root %llu of limb %u is not a primitive 2N-th root of unity "
                                   "mod %llu (psi^N must be -1)",
                                   static_cast<unsigned long long>(roots[l]), l,
                                   static_cast<unsigned long long>(q)));
            p.inv_roots[l] = ref_modinv(roots[l] % q, q);
        } else {
            p.inv_roots[l] = inv_roots ? inv_roots[l] : ref_modinv(roots[l], q);
        }
    }
    p.word = choose_word(p.moduli);
    const bool w32 = is32(p.word);
    p.limbs.resize(n_limbs);
    const uint32_t N = degree;
    const size_t entry = w32 ? 8 : 16;
    if (fwd) fwd->assign(entry * N * n_limbs, 0);
    if (inv) inv->assign(entry * N * n_limbs, 0);
    for (uint32_t l = 0; l < n_limbs; ++l) {
        const uint64_t q = p.moduli[l];
        LimbConst &c = p.limbs[l];
        std::memset(&c, 0, sizeof c);
        c.q = q;
        const uint64_t ninv = ref_modinv(degree, q) % q;
        c.ninv = ninv;
        if (w32) {
            c.one_shoup = q == 1 ? 0xFFFFFFFFull : (1ull << 32) / q;
            c.ninv_shoup = shoup32(static_cast<uint32_t>(ninv), static_cast<uint32_t>(q));
            c.barrett = q == 1 ? ~0ull
                               : static_cast<uint64_t>((static_cast<unsigned __int128>(1) << 64) / q);
        } else {
            c.one_shoup = shoup64(1, q);
            c.ninv_shoup = shoup64(ninv, q);
            const uint32_t k = 64 - static_cast<uint32_t>(__builtin_clzll(q));
            c.bk = k;
            c.barrett = static_cast<uint64_t>((static_cast<unsigned __int128>(1) << (2 * k)) / q);
        }
        for (int t = 0; t < 2; ++t) {
            std::vector<unsigned char> *dst = t == 0 ? fwd : inv;
            if (!dst) continue;
            TableGen g;
            g.init(p.logn, mode, t == 1, q, p.roots[l], p.inv_roots[l], ninv);
            unsigned char *base = dst->data() + entry * static_cast<size_t>(N) * l;
            for (uint32_t k = 1; k < N; ++k) {
                const uint64_t w = g.value(k);
                if (w32) {
                    uint32_t pair[2] = {static_cast<uint32_t>(w),
                                        shoup32(static_cast<uint32_t>(w), static_cast<uint32_t>(q))};
                    std::memcpy(base + entry * k, pair, 8);
                } else {
                    uint64_t pair[2] = {w, shoup64(w, q)};
                    std::memcpy(base + entry * k, pair, 16);
                }
            }
        }
    }
    p.table_bytes = 2ull * entry * N * n_limbs * (fast_supported(p.word, p.logn) ? 2 : 1);
    if (p.logn == 0)
        p.kind = KernelKind::Scale;
    else if (fast_supported(p.word, p.logn)) {
        p.kind = KernelKind::Cluster;
        p.cluster = fast_cluster_size(p.word, p.logn);
    } else if (p.logn <= smem_max_logn(p.word))
        p.kind = KernelKind::Smem;
    else
        p.kind = KernelKind::Global;
    return BC_OK;
}

void table_entry(const bc_plan &p, uint32_t limb, int table, uint32_t k, uint64_t *w,
                 uint64_t *wq) {
    TableGen g;
    g.init(p.logn, p.mode, table == 1, p.moduli[limb], p.roots[limb], p.inv_roots[limb],
           p.limbs[limb].ninv);
    const uint64_t v = g.value(k);
    *w = v;
    *wq = is32(p.word) ? shoup32(static_cast<uint32_t>(v), static_cast<uint32_t>(p.moduli[limb]))
                       : shoup64(v, p.moduli[limb]);
}

// ---------------------------------------------------------------- launches

namespace {

int make_args(bc_plan *p, const uint64_t *in, const uint64_t *in2, uint64_t *out,
              uint32_t batch, const bc_layout *layout, KArgs *a) {
    if (batch == 0) return fail(BC_ERR_INVALID_INPUT, "batch must be at least 1");
    if ((!in && batch) || !out) return fail(BC_ERR_INVALID_INPUT, "device pointers must not be NULL");
    std::memset(a, 0, sizeof *a);
    a->in = in;
    a->in2 = in2;
    a->out = out;
    a->poly_stride = layout ? layout->poly_stride : p->degree;
    a->limb_stride = layout ? layout->limb_stride : static_cast<int64_t>(batch) * p->degree;
    if (layout && (layout->poly_stride < 0 || layout->limb_stride < 0))
        return fail(BC_ERR_INVALID_INPUT, "layout strides must be non-negative");
    a->batch = batch;
    a->n_limbs = p->n_limbs;
    a->logn = p->logn;
    a->limbs = p->d_limbs;
    a->status = p->ctx->d_status;
    return BC_OK;
}

size_t wbytes(Word w) { return w == Word::W64 ? 8 : 4; }

// Multi-pass transform with a temporary from the context's stream-ordered
// pool: allocated and freed on `s` around the launches, so it is private to
// this call and outlives its kernels without any synchronization.
int run_global(bc_plan *p, bool gs, bool inverse, const KArgs &a, uint32_t batch, cudaStream_t s) {
    const size_t need = wbytes(p->word) * (static_cast<size_t>(batch) * p->n_limbs) << p->logn;
    void *scratch = nullptr;
    cudaError_t e = cudaMallocFromPoolAsync(&scratch, need, p->ctx->pool, s);
    if (e != cudaSuccess) return cuda_fail(e, "transform scratch");
    const int st = p->kind == KernelKind::Global ? launch_ntt_multipass(p->word, gs, inverse, a, scratch, s)
                                                 : launch_ntt_global(p->word, gs, inverse, a, scratch, s);
    e = cudaFreeAsync(scratch, s);
    if (st) return st;
    return e == cudaSuccess ? BC_OK : cuda_fail(e, "transform scratch release");
}

// The fast kernels move pairs of coefficients as 16-byte words.
bool fast_layout_ok(const KArgs &a) {
    const auto aligned = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    return aligned(a.in) && aligned(a.out) && (a.poly_stride % 2 == 0) && (a.limb_stride % 2 == 0);
}

int run_transform(bc_plan *p, bool inverse, const uint64_t *in, uint64_t *out, uint32_t batch,
                  const bc_layout *layout, cudaStream_t s) {
    KArgs a;
    int st = make_args(p, in, nullptr, out, batch, layout, &a);
    if (st) return st;
    if ((st = use_device(p->ctx))) return st;
    const bool gs = inverse && p->mode == BC_NTT_NEGACYCLIC;
    a.tw = inverse ? p->d_tw_inv : p->d_tw_fwd;
    switch (p->kind) {
    case KernelKind::Scale:
        // degree 1: both directions multiply by N^-1 = 1 (reduction mod q)
        return launch_scale(p->word, a, s);
    case KernelKind::Cluster:
        if (fast_layout_ok(a)) {
            a.tw = inverse ? p->d_tw_inv_fast : p->d_tw_fwd_fast;
            return launch_ntt_fast(p->word, gs, inverse, a, s);
        }
        if (p->logn <= smem_max_logn(p->word)) return launch_ntt_smem(p->word, gs, inverse, a, s);
        [[fallthrough]];
    case KernelKind::Global: return run_global(p, gs, inverse, a, batch, s);
    case KernelKind::Smem: return launch_ntt_smem(p->word, gs, inverse, a, s);
    default: return run_global(p, gs, inverse, a, batch, s);
    }
}

}  // namespace

int run_forward(bc_plan *p, const uint64_t *in, uint64_t *out, uint32_t batch,
                const bc_layout *layout, cudaStream_t s) {
    return run_transform(p, false, in, out, batch, layout, s);
}

int run_inverse(bc_plan *p, const uint64_t *in, uint64_t *out, uint32_t batch,
                const bc_layout *layout, cudaStream_t s) {
    return run_transform(p, true, in, out, batch, layout, s);
}

int run_pointwise(bc_plan *p, const uint64_t *a_, const uint64_t *b, uint64_t *c, uint32_t batch,
                  const bc_layout *layout, cudaStream_t s) {
    KArgs a;
    int st = make_args(p, a_, b, c, batch, layout, &a);
    if (st) return st;
    if (!b) return fail(BC_ERR_INVALID_INPUT, "device pointers must not be NULL");
    if ((st = use_device(p->ctx))) return st;
    return launch_pointwise(p->word, a, s);
}

namespace {

// How run_polymul computes a product (see there).
enum class PolymulPath { Smem, Fast, Unfused };

// The cluster kernels' product (NTT(B) into C, then one fused launch) comes
// first wherever it applies: measured on B200 (32 limbs, 2^25 words per
// operand) it is 2.5-3.7x faster than the single-CTA shared-memory kernel at
// N = 2^10..2^14, which serves cyclic plans and the layouts the cluster
// kernels cannot take.
PolymulPath polymul_path(const bc_plan *p, const KArgs &a) {
    const auto aligned = [](const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    const bool all_alias = a.in == a.out && a.in2 == a.out;
    const bool fused_mode = p->mode == BC_NTT_NEGACYCLIC || p->d_tw_gs_fast != nullptr;
    if (fused_mode && p->kind == KernelKind::Cluster && fast_layout_ok(a) &&
        aligned(a.in2) && !all_alias &&
        fast_variant_for(p->word, p->logn, false) == fast_variant_for(p->word, p->logn, true))
        return PolymulPath::Fast;
    if (p->logn >= 1 && p->logn <= polymul_smem_max_logn(p->word)) return PolymulPath::Smem;
    return PolymulPath::Unfused;
}

}  // namespace

bool polymul_allocates(bc_plan *p, const uint64_t *a_, const uint64_t *b, uint64_t *c, uint32_t batch,
                       const bc_layout *layout) {
    KArgs a;
    if (make_args(p, a_, b, c, batch, layout, &a) != BC_OK) return false;  // run_polymul fails first
    return polymul_path(p, a) == PolymulPath::Unfused;
}

namespace {

int run_polymul_impl(bc_plan *p, const uint64_t *a_, const uint64_t *b, uint64_t *c, uint32_t batch,
                     const bc_layout *layout, cudaStream_t s) {
    KArgs a;
    int st = make_args(p, a_, b, c, batch, layout, &a);
    if (st) return st;
    if (!b) return fail(BC_ERR_INVALID_INPUT, "device pointers must not be NULL");
    if ((st = use_device(p->ctx))) return st;
    const bool cyclic = p->mode == BC_NTT_CYCLIC;
    switch (polymul_path(p, a)) {
    case PolymulPath::Smem:
        a.tw = p->d_tw_fwd;
        a.tw2 = p->d_tw_inv;
        return launch_polymul_smem(p->word, cyclic, a, s);
    case PolymulPath::Fast: {
        // Fast schedules: C <- NTT(y), then one fused kernel
        // C <- INTT(NTT(x) * C), the inverse as a Gentleman-Sande network
        // (the negacyclic inverse table, or the cyclic plan's GS table).
        // The product commutes, so when A aliases C the roles swap and A's
        // transform is the one written into C.
        const uint64_t *x = a_, *y = b;
        if (x == c) std::swap(x, y);
        KArgs f = a;
        f.in = y;
        f.in2 = nullptr;
        f.tw = p->d_tw_fwd_fast;
        if ((st = launch_ntt_fast(p->word, false, false, f, s))) return st;
        a.in = x;
        a.in2 = c;
        a.tw = p->d_tw_fwd_fast;
        a.tw2 = cyclic ? p->d_tw_gs_fast : p->d_tw_inv_fast;
        return launch_polymul_fast(p->word, a, s);
    }
    default: break;
    }
    // Unfused fallback above the fused size: forward both operands into a
    // temporary compact buffer, multiply, inverse into the caller's layout.
    const bool caller_compact =
        !layout || (layout->poly_stride == p->degree &&
                    layout->limb_stride == static_cast<int64_t>(batch) * p->degree);
    if (!caller_compact)
        return fail(BC_ERR_UNSUPPORTED, "polymul above the fused size needs the default layout");
    // The temporary comes from the context's stream-ordered pool and is
    // released on the same stream after the last launch that reads it, so
    // the call neither synchronizes nor frees memory another stream uses.
    const size_t words = (static_cast<size_t>(batch) * p->n_limbs) << p->logn;
    void *raw = nullptr;
    cudaError_t e = cudaMallocFromPoolAsync(&raw, 2 * words * sizeof(uint64_t), p->ctx->pool, s);
    if (e != cudaSuccess) return cuda_fail(e, "polymul scratch allocation");
    uint64_t *tmp = static_cast<uint64_t *>(raw);
    int r = run_transform(p, false, a_, tmp, batch, layout, s);
    if (!r) r = run_transform(p, false, b, tmp + words, batch, layout, s);
    if (!r) r = run_pointwise(p, tmp, tmp + words, tmp, batch, layout, s);
    if (!r) r = run_transform(p, true, tmp, c, batch, layout, s);
    e = cudaFreeAsync(raw, s);
    if (r) return r;
    return e == cudaSuccess ? BC_OK : cuda_fail(e, "polymul scratch release");
}

}  // namespace

int run_polymul(bc_plan *p, const uint64_t *a_, const uint64_t *b, uint64_t *c, uint32_t batch,
                const bc_layout *layout, cudaStream_t s) {
    return run_polymul_impl(p, a_, b, c, batch, layout, s);
}

int cached_plan(bc_ctx *ctx, uint32_t degree, uint64_t modulus, uint64_t root, uint64_t inv_root,
                int mode, std::shared_ptr<bc_plan> *out) {
    std::lock_guard<std::mutex> lk(ctx->cache_mu);
    for (auto it = ctx->cache.begin(); it != ctx->cache.end(); ++it) {
        if (it->degree == degree && it->modulus == modulus && it->root == root &&
            it->inv_root == inv_root && it->mode == mode) {
            ctx->cache.splice(ctx->cache.begin(), ctx->cache, it);
            *out = it->plan;
            return BC_OK;
        }
    }
    bc_plan *p = nullptr;
    const int st = bc_plan_create(ctx, degree, 1, &modulus, &root,
                                  mode == BC_NTT_CYCLIC ? &inv_root : nullptr, mode, &p);
    if (st) return st;
    std::shared_ptr<bc_plan> sp(p, [](bc_plan *q) { bc_plan_destroy(q); });
    ctx->cache.push_front({degree, modulus, root, inv_root, mode, sp});
    // an evicted plan still in use by another caller goes when that caller ends
    while (ctx->cache.size() > 32) ctx->cache.pop_back();
    *out = std::move(sp);
    return BC_OK;
}

}  // namespace bc

using namespace bc;

// ================================================================== C ABI

extern "C" {

const char *bc_last_error(void) { return bc::last_error_cstr(); }

int bc_abi_version(void) { return BC_ABI_VERSION; }

int bc_device_count(int *count) {
    if (!count) return fail(BC_ERR_INVALID_INPUT, "count must not be NULL");
    int n = 0;
    const cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
        *count = 0;
        return cuda_fail(e, "cudaGetDeviceCount");
    }
    *count = n;
    return BC_OK;
}

int bc_ctx_create(int device, bc_ctx **out) {
    if (!out) return fail(BC_ERR_INVALID_INPUT, "out must not be NULL");
    *out = nullptr;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
    if (device < 0 || device >= n)
        return fail(BC_ERR_DEVICE_NOT_AVAILABLE, format("device %d not present (%d visible)", device, n));
    if ((e = cudaSetDevice(device)) != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    cudaDeviceProp prop;
    if ((e = cudaGetDeviceProperties(&prop, device)) != cudaSuccess)
        return cuda_fail(e, "cudaGetDeviceProperties");
    if (prop.major != 10)
        return fail(BC_ERR_UNSUPPORTED,
                    format("device %d is sm_%d%d; this library is built for sm_100a (B200)", device,
                           prop.major, prop.minor));
    auto *c = new bc_ctx();
    c->device = device;
    if ((e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking)) != cudaSuccess) {
        delete c;
        return cuda_fail(e, "cudaStreamCreate");
    }
    // status word: mapped page-locked host memory (see bc_kernels.hpp)
    void *hs = nullptr, *ds = nullptr;
    if ((e = cudaHostAlloc(&hs, sizeof(uint32_t), cudaHostAllocMapped | cudaHostAllocPortable)) != cudaSuccess ||
        (e = cudaHostGetDevicePointer(&ds, hs, 0)) != cudaSuccess) {
        if (hs) cudaFreeHost(hs);
        cudaStreamDestroy(c->stream);
        delete c;
        return cuda_fail(e, "status word allocation");
    }
    c->h_status = static_cast<uint32_t *>(hs);
    c->d_status = static_cast<uint32_t *>(ds);
    *c->h_status = 0;
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = device;
    if ((e = cudaMemPoolCreate(&c->pool, &props)) != cudaSuccess) {
        cudaFreeHost(c->h_status);
        cudaStreamDestroy(c->stream);
        delete c;
        return cuda_fail(e, "memory pool creation");
    }
    // keep freed temporaries in the pool instead of returning them at every
    // synchronization (the pool belongs to this context only)
    uint64_t keep = UINT64_MAX;
    cudaMemPoolSetAttribute(c->pool, cudaMemPoolAttrReleaseThreshold, &keep);
    *out = c;
    return BC_OK;
}

int bc_ctx_destroy(bc_ctx *ctx) {
    if (!ctx) return BC_OK;
    use_device(ctx);
    cudaStreamSynchronize(ctx->stream);
    ctx->cache.clear();  // destroys the cached plans (no caller holds one now)
    cudaFreeHost(ctx->h_status);  // d_status is its device mapping
    cudaStreamDestroy(ctx->stream);
    // returns at once; the pool goes once its last stream-ordered free completes
    if (ctx->pool) cudaMemPoolDestroy(ctx->pool);
    delete ctx;
    return BC_OK;
}

int bc_ctx_device(const bc_ctx *ctx, int *device) {
    if (!ctx || !device) return fail(BC_ERR_INVALID_INPUT, "NULL argument");
    *device = ctx->device;
    return BC_OK;
}

int bc_ctx_stream(bc_ctx *ctx, void **stream) {
    if (!ctx || !stream) return fail(BC_ERR_INVALID_INPUT, "NULL argument");
    *stream = ctx->stream;
    return BC_OK;
}

int bc_ctx_sync(bc_ctx *ctx) {
    if (!ctx) return fail(BC_ERR_INVALID_INPUT, "NULL context");
    int st = use_device(ctx);
    return st ? st : ctx_sync(ctx);
}

// Buffers come from the context's memory pool, which keeps freed memory for
// reuse: a reference-op call that allocates its output (FheNtt::execute
// returns a new tensor) then costs no driver allocation.  The guarantees of
// cudaMalloc / cudaFree stay: the memory is usable by every stream when
// bc_buf_alloc returns (the context stream is idle, or is waited for), and
// bc_buf_free first waits for all work on the device, as cudaFree does.
int bc_buf_alloc(bc_ctx *ctx, size_t bytes, void **dptr) {
    if (!ctx || !dptr) return fail(BC_ERR_INVALID_INPUT, "NULL argument");
    *dptr = nullptr;
    int st = use_device(ctx);
    if (st) return st;
    cudaError_t e = cudaMallocFromPoolAsync(dptr, bytes ? bytes : 1, ctx->pool, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "device buffer allocation");
    if (cudaStreamQuery(ctx->stream) != cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    return e == cudaSuccess ? BC_OK : cuda_fail(e, "device buffer allocation");
}

int bc_buf_free(bc_ctx *ctx, void *dptr) {
    if (!ctx) return fail(BC_ERR_INVALID_INPUT, "NULL context");
    if (!dptr) return BC_OK;
    use_device(ctx);
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaFreeAsync(dptr, ctx->stream);
    return e == cudaSuccess ? BC_OK : cuda_fail(e, "device buffer release");
}

static int copy_sync(bc_ctx *ctx, void *dst, const void *src, size_t bytes, cudaMemcpyKind k) {
    if (!ctx || (!dst && bytes) || (!src && bytes)) return fail(BC_ERR_INVALID_INPUT, "NULL argument");
    int st = use_device(ctx);
    if (st) return st;
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, k, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    return e == cudaSuccess ? BC_OK : cuda_fail(e, "cudaMemcpy");
}

int bc_buf_h2d(bc_ctx *ctx, void *dst, const void *src, size_t bytes) {
    return copy_sync(ctx, dst, src, bytes, cudaMemcpyHostToDevice);
}

int bc_buf_d2h(bc_ctx *ctx, void *dst, const void *src, size_t bytes) {
    return copy_sync(ctx, dst, src, bytes, cudaMemcpyDeviceToHost);
}

static int copy_async(bc_ctx *ctx, void *dst, const void *src, size_t bytes, cudaMemcpyKind k,
                      void *stream) {
    if (!ctx || (!dst && bytes) || (!src && bytes)) return fail(BC_ERR_INVALID_INPUT, "NULL argument");
    int st = use_device(ctx);
    if (st) return st;
    const cudaError_t e =
        cudaMemcpyAsync(dst, src, bytes, k, stream ? static_cast<cudaStream_t>(stream) : ctx->stream);
    return e == cudaSuccess ? BC_OK : cuda_fail(e, "cudaMemcpyAsync");
}

int bc_buf_h2d_async(bc_ctx *ctx, void *dst, const void *src, size_t bytes, void *stream) {
    return copy_async(ctx, dst, src, bytes, cudaMemcpyHostToDevice, stream);
}

int bc_buf_d2h_async(bc_ctx *ctx, void *dst, const void *src, size_t bytes, void *stream) {
    return copy_async(ctx, dst, src, bytes, cudaMemcpyDeviceToHost, stream);
}

int bc_host_alloc(size_t bytes, void **hptr) {
    if (!hptr) return fail(BC_ERR_INVALID_INPUT, "NULL argument");
    const cudaError_t e = cudaMallocHost(hptr, bytes ? bytes : 1);
    return e == cudaSuccess ? BC_OK : cuda_fail(e, "cudaMallocHost");
}

int bc_host_free(void *hptr) {
    if (!hptr) return BC_OK;
    const cudaError_t e = cudaFreeHost(hptr);
    return e == cudaSuccess ? BC_OK : cuda_fail(e, "cudaFreeHost");
}

int bc_plan_create(bc_ctx *ctx, uint32_t degree, uint32_t n_limbs, const uint64_t *moduli,
                   const uint64_t *roots, const uint64_t *inv_roots, int mode, bc_plan **out) {
    if (!ctx || !out) return fail(BC_ERR_INVALID_INPUT, "NULL argument");
    *out = nullptr;
    auto *p = new bc_plan();
    p->ctx = ctx;
    std::vector<unsigned char> fwd, inv;
    int st = plan_build_host(*p, degree, n_limbs, moduli, roots, inv_roots, mode, &fwd, &inv);
    if (st) {
        delete p;
        return st;
    }
    if ((st = use_device(ctx))) {
        delete p;
        return st;
    }
    // the multi-pass kernels (every plan above the cluster kernels) read the
    // stages below their TOP pass permuted
    if (p->kind == KernelKind::Global) {
        const size_t entry = p->word == Word::W64 ? 16 : 8;
        const uint64_t N = degree;
        const uint32_t top_lo = multipass_top_lo(p->word, p->logn);
        std::vector<unsigned char> tmp(entry * N);
        for (std::vector<unsigned char> *t : {&fwd, &inv}) {
            for (uint32_t l = 0; l < n_limbs; ++l) {
                unsigned char *base = t->data() + entry * N * l;
                std::memcpy(tmp.data(), base, tmp.size());
                for (uint64_t k = 1; k < N; ++k)
                    std::memcpy(base + entry * multipass_table_index(p->logn, top_lo, k), tmp.data() + entry * k,
                                entry);
            }
        }
    }
    // the fast kernels read each direction's table in their own layout
    std::vector<unsigned char> fwd_fast, inv_fast, gs_fast;
    if (p->kind == KernelKind::Cluster) {
        const size_t entry = p->word == Word::W64 ? 16 : 8;
        const int pair = p->word == Word::W64 ? 1 : 2;
        const uint64_t N = degree;
        const bool w32 = p->word != Word::W64;
        const int vf = fast_variant_for(p->word, p->logn, false), vi = fast_variant_for(p->word, p->logn, true);
        const bool gs = p->mode == BC_NTT_CYCLIC && vf == vi && cyclic_roots_primitive(*p);
        for (int t = 0; t < (gs ? 3 : 2); ++t) {
            std::vector<unsigned char> gs_plain;
            if (t == 2) {  // cyclic inverse in Gentleman-Sande form
                gs_plain.assign(inv.size(), 0);
                for (uint32_t l = 0; l < n_limbs; ++l) {
                    TableGen g;
                    const uint64_t q = p->moduli[l];
                    g.init(p->logn, p->mode, true, q, p->roots[l], p->inv_roots[l], p->limbs[l].ninv, true);
                    unsigned char *base = gs_plain.data() + entry * N * l;
                    for (uint64_t k = 1; k < N; ++k) {
                        const uint64_t w = g.value(static_cast<uint32_t>(k));
                        if (w32) {
                            uint32_t pr[2] = {static_cast<uint32_t>(w), shoup32(static_cast<uint32_t>(w), static_cast<uint32_t>(q))};
                            std::memcpy(base + entry * k, pr, 8);
                        } else {
                            uint64_t pr[2] = {w, shoup64(w, q)};
                            std::memcpy(base + entry * k, pr, 16);
                        }
                    }
                }
            }
            const std::vector<unsigned char> &src = t == 0 ? fwd : t == 1 ? inv : gs_plain;
            std::vector<unsigned char> &dst = t == 0 ? fwd_fast : t == 1 ? inv_fast : gs_fast;
            dst.assign(src.size(), 0);
            const int V = t == 0 ? vf : vi;
            std::vector<uint64_t> map(N);
            for (uint64_t k = 1; k < N; ++k) map[k] = fast_table_index(p->logn, V, k, pair);
            for (uint32_t l = 0; l < n_limbs; ++l) {
                const unsigned char *sb = src.data() + entry * N * l;
                unsigned char *db = dst.data() + entry * N * l;
                for (uint64_t k = 1; k < N; ++k) std::memcpy(db + entry * map[k], sb + entry * k, entry);
            }
        }
        p->table_bytes += gs_fast.size();
    }
    std::vector<CoeffConst> coeff(n_limbs);
    for (uint32_t l = 0; l < n_limbs; ++l) coeff[l] = coeff_const(p->moduli[l]);
    cudaError_t e = cudaMalloc(&p->d_limbs, sizeof(LimbConst) * n_limbs);
    if (e == cudaSuccess) e = cudaMalloc(&p->d_coeff, sizeof(CoeffConst) * n_limbs);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(p->d_coeff, coeff.data(), sizeof(CoeffConst) * n_limbs, cudaMemcpyHostToDevice,
                            ctx->stream);
    if (e == cudaSuccess) e = cudaMalloc(&p->d_tw_fwd, fwd.size());
    if (e == cudaSuccess) e = cudaMalloc(&p->d_tw_inv, inv.size());
    if (e == cudaSuccess && !fwd_fast.empty()) e = cudaMalloc(&p->d_tw_fwd_fast, fwd_fast.size());
    if (e == cudaSuccess && !inv_fast.empty()) e = cudaMalloc(&p->d_tw_inv_fast, inv_fast.size());
    if (e == cudaSuccess && !fwd_fast.empty())
        e = cudaMemcpyAsync(p->d_tw_fwd_fast, fwd_fast.data(), fwd_fast.size(), cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess && !inv_fast.empty())
        e = cudaMemcpyAsync(p->d_tw_inv_fast, inv_fast.data(), inv_fast.size(), cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess && !gs_fast.empty()) e = cudaMalloc(&p->d_tw_gs_fast, gs_fast.size());
    if (e == cudaSuccess && !gs_fast.empty())
        e = cudaMemcpyAsync(p->d_tw_gs_fast, gs_fast.data(), gs_fast.size(), cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(p->d_limbs, p->limbs.data(), sizeof(LimbConst) * n_limbs,
                            cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(p->d_tw_fwd, fwd.data(), fwd.size(), cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(p->d_tw_inv, inv.data(), inv.size(), cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) {
        st = cuda_fail(e, "plan upload");
        bc_plan_destroy(p);
        return st;
    }
    *out = p;
    return BC_OK;
}

int bc_plan_destroy(bc_plan *p) {
    if (!p) return BC_OK;
    use_device(p->ctx);
    cudaStreamSynchronize(p->ctx->stream);
    cudaFree(p->d_limbs);
    cudaFree(p->d_coeff);
    cudaFree(p->d_tw_fwd);
    cudaFree(p->d_tw_inv);
    cudaFree(p->d_tw_fwd_fast);
    cudaFree(p->d_tw_inv_fast);
    cudaFree(p->d_tw_gs_fast);
    delete p;
    return BC_OK;
}

int bc_plan_info_get(const bc_plan *p, bc_plan_info *out) {
    if (!p || !out) return fail(BC_ERR_INVALID_INPUT, "NULL argument");
    out->degree = p->degree;
    out->n_limbs = p->n_limbs;
    out->mode = p->mode;
    out->word_bits = p->word == Word::W64 ? 64 : 32;
    out->kernel_kind = static_cast<int32_t>(p->kind);
    out->cluster_size = p->cluster;
    out->table_bytes = p->table_bytes;
    return BC_OK;
}

static cudaStream_t pick_stream(bc_plan *p, void *stream) {
    return stream ? static_cast<cudaStream_t>(stream) : p->ctx->stream;
}

int bc_ntt_forward(bc_plan *p, const uint64_t *in, uint64_t *out, uint32_t batch,
                   const bc_layout *layout, void *stream) {
    if (!p) return fail(BC_ERR_INVALID_INPUT, "NULL plan");
    return run_forward(p, in, out, batch, layout, pick_stream(p, stream));
}

int bc_ntt_inverse(bc_plan *p, const uint64_t *in, uint64_t *out, uint32_t batch,
                   const bc_layout *layout, void *stream) {
    if (!p) return fail(BC_ERR_INVALID_INPUT, "NULL plan");
    return run_inverse(p, in, out, batch, layout, pick_stream(p, stream));
}

int bc_pointwise_mul(bc_plan *p, const uint64_t *a, const uint64_t *b, uint64_t *c, uint32_t batch,
                     const bc_layout *layout, void *stream) {
    if (!p) return fail(BC_ERR_INVALID_INPUT, "NULL plan");
    return run_pointwise(p, a, b, c, batch, layout, pick_stream(p, stream));
}

static int run_coeff(bc_plan *p, int op, const uint64_t *a_, const uint64_t *b, uint64_t *c,
                     uint32_t batch, const bc_layout *layout, void *stream) {
    if (!p) return fail(BC_ERR_INVALID_INPUT, "NULL plan");
    KArgs a;
    int st = make_args(p, a_, b, c, batch, layout, &a);
    if (st) return st;
    if (!b) return fail(BC_ERR_INVALID_INPUT, "device pointers must not be NULL");
    if ((st = use_device(p->ctx))) return st;
    return launch_coeff_op(op, a, p->degree, p->d_coeff, CoeffConst{}, pick_stream(p, stream));
}

int bc_poly_add(bc_plan *p, const uint64_t *a, const uint64_t *b, uint64_t *c, uint32_t batch,
                const bc_layout *layout, void *stream) {
    return run_coeff(p, kCoeffAdd, a, b, c, batch, layout, stream);
}

int bc_poly_sub(bc_plan *p, const uint64_t *a, const uint64_t *b, uint64_t *c, uint32_t batch,
                const bc_layout *layout, void *stream) {
    return run_coeff(p, kCoeffSub, a, b, c, batch, layout, stream);
}

int bc_poly_mul(bc_plan *p, const uint64_t *a, const uint64_t *b, uint64_t *c, uint32_t batch,
                const bc_layout *layout, void *stream) {
    return run_coeff(p, kCoeffMul, a, b, c, batch, layout, stream);
}

// The pointwise step of the fused transforms as its own launch: the product,
// or the exact sum / difference of the inputs reduced mod q.
static int pointwise_step(bc_plan *p, uint32_t op, const uint64_t *x, const uint64_t *y, uint64_t *out,
                          uint32_t batch, const bc_layout *layout, cudaStream_t s) {
    if (op == kFuseMul) return run_pointwise(p, x, y, out, batch, layout, s);
    KArgs a;
    const int st = make_args(p, x, y, out, batch, layout, &a);
    if (st) return st;
    return launch_coeff_op(op == kFuseAdd ? kCoeffAddExact : kCoeffSubExact, a, p->degree, p->d_coeff,
                           CoeffConst{}, s, p->word != Word::W64);
}

// Transform fused with a pointwise step (kFuseMul / kFuseAdd / kFuseSub):
// one launch on the fast kernels (negacyclic plans, 16-byte aligned
// operands, even strides); otherwise a transform launch and a pointwise
// launch with the same result.
static int run_ntt_fused(bc_plan *p, bool inverse, uint32_t op, const uint64_t *a_, const uint64_t *b,
                         uint64_t *c, uint32_t batch, const bc_layout *layout, void *stream) {
    if (!p) return fail(BC_ERR_INVALID_INPUT, "NULL plan");
    KArgs a;
    int st = make_args(p, a_, b, c, batch, layout, &a);
    if (st) return st;
    if (!b) return fail(BC_ERR_INVALID_INPUT, "device pointers must not be NULL");
    if ((st = use_device(p->ctx))) return st;
    const cudaStream_t s = pick_stream(p, stream);
    const bool b_aligned = (reinterpret_cast<uintptr_t>(b) & 15u) == 0;
    if (p->kind == KernelKind::Cluster && p->mode == BC_NTT_NEGACYCLIC && fast_layout_ok(a) && b_aligned) {
        a.tw = inverse ? p->d_tw_inv_fast : p->d_tw_fwd_fast;
        a.op = op;
        return launch_ntt_mul_fast(p->word, inverse, a, s);
    }
    if (inverse) {  // C = A^ op B^ elementwise (any aliasing), then the inverse in place
        if ((st = pointwise_step(p, op, a_, b, c, batch, layout, s))) return st;
        return run_inverse(p, c, c, batch, layout, s);
    }
    if (c != b) {
        if ((st = run_forward(p, a_, c, batch, layout, s))) return st;
        return pointwise_step(p, op, c, b, c, batch, layout, s);
    }
    // C is B^: the forward needs a buffer of its own, laid out like C
    const int64_t ls = a.limb_stride, ps = a.poly_stride;
    const size_t extent = static_cast<size_t>(ls) * (p->n_limbs - 1) + static_cast<size_t>(ps) * (batch - 1) + p->degree;
    void *tmp = nullptr;
    cudaError_t e = cudaMallocFromPoolAsync(&tmp, extent * sizeof(uint64_t), p->ctx->pool, s);
    if (e != cudaSuccess) return cuda_fail(e, "fused-transform temporary");
    uint64_t *t = static_cast<uint64_t *>(tmp);
    st = run_forward(p, a_, t, batch, layout, s);
    if (!st) st = pointwise_step(p, op, t, b, c, batch, layout, s);
    e = cudaFreeAsync(tmp, s);
    if (st) return st;
    return e == cudaSuccess ? BC_OK : cuda_fail(e, "fused-transform temporary release");
}

int bc_ntt_forward_mul(bc_plan *p, const uint64_t *a, const uint64_t *b_hat, uint64_t *c, uint32_t batch,
                       const bc_layout *layout, void *stream) {
    return run_ntt_fused(p, false, kFuseMul, a, b_hat, c, batch, layout, stream);
}

int bc_ntt_inverse_mul(bc_plan *p, const uint64_t *a_hat, const uint64_t *b_hat, uint64_t *c, uint32_t batch,
                       const bc_layout *layout, void *stream) {
    return run_ntt_fused(p, true, kFuseMul, a_hat, b_hat, c, batch, layout, stream);
}

int bc_ntt_forward_add(bc_plan *p, const uint64_t *a, const uint64_t *b_hat, uint64_t *c, uint32_t batch,
                       const bc_layout *layout, void *stream) {
    return run_ntt_fused(p, false, kFuseAdd, a, b_hat, c, batch, layout, stream);
}

int bc_ntt_forward_sub(bc_plan *p, const uint64_t *a, const uint64_t *b_hat, uint64_t *c, uint32_t batch,
                       const bc_layout *layout, void *stream) {
    return run_ntt_fused(p, false, kFuseSub, a, b_hat, c, batch, layout, stream);
}

int bc_ntt_inverse_add(bc_plan *p, const uint64_t *a_hat, const uint64_t *b_hat, uint64_t *c, uint32_t batch,
                       const bc_layout *layout, void *stream) {
    return run_ntt_fused(p, true, kFuseAdd, a_hat, b_hat, c, batch, layout, stream);
}

int bc_ntt_inverse_sub(bc_plan *p, const uint64_t *a_hat, const uint64_t *b_hat, uint64_t *c, uint32_t batch,
                       const bc_layout *layout, void *stream) {
    return run_ntt_fused(p, true, kFuseSub, a_hat, b_hat, c, batch, layout, stream);
}

int bc_polymul(bc_plan *p, const uint64_t *a, const uint64_t *b, uint64_t *c, uint32_t batch,
               const bc_layout *layout, void *stream) {
    if (!p) return fail(BC_ERR_INVALID_INPUT, "NULL plan");
    return run_polymul(p, a, b, c, batch, layout, pick_stream(p, stream));
}

int bc_automorphism(bc_plan *p, const uint64_t *in, uint64_t *out, uint32_t batch, const bc_layout *layout,
                    uint32_t galois, void *stream) {
    if (!p) return fail(BC_ERR_INVALID_INPUT, "NULL plan");
    if ((galois & 1u) == 0 || galois >= 2ull * p->degree)
        return fail(BC_ERR_INVALID_INPUT,
                    format("galois element %u must be odd and below 2N = %llu", galois,
                           static_cast<unsigned long long>(2ull * p->degree)));
    KArgs a;
    int st = make_args(p, in, nullptr, out, batch, layout, &a);
    if (st) return st;
    if (in == out) return fail(BC_ERR_INVALID_INPUT, "input and output must be different buffers");
    if ((st = use_device(p->ctx))) return st;
    return launch_automorphism(a, galois, p->d_coeff, 0, pick_stream(p, stream));
}

int bc_modulus_switch(bc_ctx *ctx, const uint64_t *in, uint64_t *out, size_t count, uint64_t modulus_old,
                      uint64_t modulus_new, void *stream) {
    if (!ctx || ((!in || !out) && count)) return fail(BC_ERR_INVALID_INPUT, "NULL argument");
    if (modulus_new >= modulus_old)
        return fail(BC_ERR_INVALID_INPUT, format("New modulus (%llu) must be < old modulus (%llu)",
                                                 static_cast<unsigned long long>(modulus_new),
                                                 static_cast<unsigned long long>(modulus_old)));
    int st = use_device(ctx);
    if (st) return st;
    return launch_modulus_switch(in, out, count, modswitch_const(modulus_old, modulus_new),
                                 stream ? static_cast<cudaStream_t>(stream) : ctx->stream);
}

int bc_decompose(bc_ctx *ctx, const uint64_t *in, uint64_t *out, size_t count, uint32_t base, uint32_t levels,
                 void *stream) {
    if (!ctx || ((!in || !out) && count)) return fail(BC_ERR_INVALID_INPUT, "NULL argument");
    if (base < 2 || base > (1u << 24))
        return fail(BC_ERR_INVALID_INPUT, format("Decomposition base must be in [2, 2^24], got %u", base));
    if (levels == 0 || levels > 32)
        return fail(BC_ERR_INVALID_INPUT, format("Decomposition levels must be in [1, 32], got %u", levels));
    const uintptr_t ib = reinterpret_cast<uintptr_t>(in), ob = reinterpret_cast<uintptr_t>(out);
    if (count && ib < ob + count * levels * sizeof(uint64_t) && ob < ib + count * sizeof(uint64_t))
        return fail(BC_ERR_INVALID_INPUT, "input and output must not overlap");
    int st = use_device(ctx);
    if (st) return st;
    return launch_decompose(in, out, count, base, levels, stream ? static_cast<cudaStream_t>(stream) : ctx->stream);
}

int bc_fill_uniform(bc_plan *p, uint64_t *out, uint32_t batch, const bc_layout *layout, uint64_t seed,
                    uint64_t first_poly, uint64_t total_polys, void *stream) {
    if (!p) return fail(BC_ERR_INVALID_INPUT, "NULL plan");
    KArgs a;
    std::memset(&a, 0, sizeof a);
    if (!out || batch == 0) return fail(BC_ERR_INVALID_INPUT, "empty fill");
    a.out = out;
    a.poly_stride = layout ? layout->poly_stride : p->degree;
    a.limb_stride = layout ? layout->limb_stride : static_cast<int64_t>(batch) * p->degree;
    a.batch = batch;
    a.n_limbs = p->n_limbs;
    a.logn = p->logn;
    a.limbs = p->d_limbs;
    int st = use_device(p->ctx);
    if (st) return st;
    return launch_fill_uniform(a, seed, first_poly, total_polys, pick_stream(p, stream));
}

int bc_digest(bc_ctx *ctx, const uint64_t *in, size_t count, uint64_t first_index, uint64_t *out,
              void *stream) {
    if (!ctx || !out || (!in && count)) return fail(BC_ERR_INVALID_INPUT, "NULL argument");
    int st = use_device(ctx);
    if (st) return st;
    return launch_digest(in, count, first_index, out,
                         stream ? static_cast<cudaStream_t>(stream) : ctx->stream);
}

int bc_partition(uint64_t units, uint32_t shards, uint32_t shard, uint64_t *begin, uint64_t *count) {
    if (!begin || !count) return fail(BC_ERR_INVALID_INPUT, "NULL argument");
    if (shards == 0 || shard >= shards)
        return fail(BC_ERR_INVALID_INPUT, format("shard %u out of range for %u shards", shard, shards));
    const uint64_t base = units / shards, extra = units % shards;
    *count = base + (shard < extra ? 1 : 0);
    *begin = shard * base + (shard < extra ? shard : extra);
    return BC_OK;
}

uint64_t bc_ntt_prime(uint32_t bits, uint32_t degree, uint32_t index) {
    return ntt_prime(bits, degree, index);
}

uint64_t bc_negacyclic_root(uint64_t modulus, uint32_t degree) {
    if (modulus < 3 || degree == 0 || (modulus - 1) % (2ull * degree) != 0 || !is_prime(modulus)) return 0;
    const uint64_t g = smallest_generator(modulus);
    return powmod(g, (modulus - 1) / (2ull * degree), modulus);
}

int bc_debug_twiddle(uint32_t degree, uint64_t modulus, uint64_t root, uint64_t inv_root, int mode,
                     int table, uint32_t k, uint64_t *w, uint64_t *w_shoup) {
    if (!w || !w_shoup) return fail(BC_ERR_INVALID_INPUT, "NULL argument");
    bc_plan p;
    int st = plan_build_host(p, degree, 1, &modulus, &root,
                             mode == BC_NTT_CYCLIC ? &inv_root : nullptr, mode, nullptr, nullptr);
    if (st) return st;
    if (k == 0 || k >= degree) return fail(BC_ERR_INVALID_INPUT, "entry index out of range");
    table_entry(p, 0, table, k, w, w_shoup);
    return BC_OK;
}

}  // extern "C"
