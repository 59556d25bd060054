// bc_static_scratch.cu -- bc_polymul_static_scratch: the NTT-based
// polynomial product without any device allocation.
//
// On its unfused path (N >= 2^18, cyclic plans with a non-primitive root
// above the fused size, layouts the fused kernels cannot take) bc_polymul
// runs forward(A) and forward(B) into a temporary, multiplies, and runs the
// inverse; it takes that temporary from the context's stream-ordered memory
// pool on every call, which grows the pool with fresh device memory when it
// holds none free.  Some callers cannot allocate during the call:
//   - processes whose device memory was reserved up front by another
//     allocator (a framework's caching pool holding the free memory), where
//     the driver has nothing left to hand out;
//   - serving loops under a fixed device-memory budget that must not grow
//     once they run.
// This entry point keeps the temporary in one fixed buffer per device in the
// library's static device memory instead, so it allocates nothing and does
// not synchronize.  The price is a size limit and a shared buffer: calls that
// overlap in time on one GPU race on it (see barracuda_fhe.h).
#include <cstdint>
#include <cstring>

#include <cuda_runtime.h>

#include "bc_common.hpp"
#include "bc_kernels.hpp"
#include "bc_runtime.hpp"

namespace bc {
namespace {

constexpr size_t kMaxCoeffs = BC_POLYMUL_STATIC_MAX_COEFFS;  // per operand
constexpr int kMaxDevices = 64;

// Two regions of kMaxCoeffs u64 words (32 MiB in all): [0, kMaxCoeffs) holds
// NTT(B) in the caller's compact layout, [kMaxCoeffs, 2 kMaxCoeffs) is the
// working area of the multi-pass global-memory transform when a transform
// has to take that path (at most 8 bytes per coefficient).  Every word is
// written before it is read, so nothing here needs to start at zero.
static __device__ __align__(256) uint64_t g_polymul_scratch[2 * kMaxCoeffs];

// Device address of the static buffer on the current device (`device`).
// Looked up on every call rather than cached: after a device reset the
// driver reloads the module and the buffer may move, and the lookup is cheap
// once the module is loaded.  The first lookup on a device may make the
// driver load this translation unit's device module; that is the set-up the
// first call does.
int scratch_address(int device, uint64_t **out) {
    if (device < 0 || device >= kMaxDevices)
        return fail(BC_ERR_UNSUPPORTED,
                    format("bc_polymul_static_scratch supports device ordinals below %d, got %d",
                           kMaxDevices, device));
    void *ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_polymul_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(polymul static scratch)");
    *out = static_cast<uint64_t *>(ptr);
    return BC_OK;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// One transform of `batch` polynomials per limb in the compact layout, with
// the kernel choice of the plan's own transforms; the global-memory path
// works in `glb` instead of the plan's lazily allocated scratch.
int transform(bc_plan *p, bool inverse, const uint64_t *in, uint64_t *out, uint32_t batch,
              void *glb, cudaStream_t s) {
    KArgs a;
    std::memset(&a, 0, sizeof a);
    a.in = in;
    a.out = out;
    a.poly_stride = p->degree;
    a.limb_stride = static_cast<int64_t>(batch) * p->degree;
    a.batch = batch;
    a.n_limbs = p->n_limbs;
    a.logn = p->logn;
    a.limbs = p->d_limbs;
    a.status = p->ctx->d_status;
    const bool gs = inverse && p->mode == BC_NTT_NEGACYCLIC;
    a.tw = inverse ? p->d_tw_inv : p->d_tw_fwd;
    const bool even = p->degree % 2 == 0;
    switch (p->kind) {
    case KernelKind::Scale: return launch_scale(p->word, a, s);
    case KernelKind::Cluster:
        if (aligned16(in) && aligned16(out) && even) {
            a.tw = inverse ? p->d_tw_inv_fast : p->d_tw_fwd_fast;
            return launch_ntt_fast(p->word, gs, inverse, a, s);
        }
        if (p->logn <= smem_max_logn(p->word)) return launch_ntt_smem(p->word, gs, inverse, a, s);
        return launch_ntt_global(p->word, gs, inverse, a, glb, s);
    case KernelKind::Smem: return launch_ntt_smem(p->word, gs, inverse, a, s);
    default: return launch_ntt_multipass(p->word, gs, inverse, a, glb, s);
    }
}

}  // namespace
}  // namespace bc

using namespace bc;

extern "C" int bc_polymul_static_scratch(bc_plan *p, const uint64_t *a, const uint64_t *b,
                                         uint64_t *c, uint32_t batch, const bc_layout *layout,
                                         void *stream) {
    if (!p) return fail(BC_ERR_INVALID_INPUT, "NULL plan");
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : p->ctx->stream;
    // Where bc_polymul needs no temporary (its fused kernels), it is the product.
    if (!polymul_allocates(p, a, b, c, batch, layout)) return run_polymul(p, a, b, c, batch, layout, s);
    if (batch == 0) return fail(BC_ERR_INVALID_INPUT, "batch must be at least 1");
    if (!a || !b || !c) return fail(BC_ERR_INVALID_INPUT, "device pointers must not be NULL");
    if (layout && (layout->poly_stride != p->degree ||
                   layout->limb_stride != static_cast<int64_t>(batch) * p->degree))
        return fail(BC_ERR_UNSUPPORTED, "polymul above the fused size needs the default layout");
    const size_t coeffs = (static_cast<size_t>(batch) * p->n_limbs) << p->logn;
    if (coeffs > kMaxCoeffs)
        return fail(BC_ERR_INVALID_INPUT,
                    format("bc_polymul_static_scratch: batch * n_limbs * N = %zu coefficients exceeds "
                           "the static scratch limit of %zu (use bc_polymul or split the batch)",
                           coeffs, kMaxCoeffs));
    int st = use_device(p->ctx);
    if (st) return st;
    uint64_t *scratch = nullptr;
    if ((st = scratch_address(p->ctx->device, &scratch))) return st;
    uint64_t *nb = scratch;              // NTT(B), compact layout
    void *glb = scratch + kMaxCoeffs;    // global-path working area
    // B first, so that C may alias A or B.
    if ((st = transform(p, false, b, nb, batch, glb, s))) return st;
    if ((st = transform(p, false, a, c, batch, glb, s))) return st;
    if ((st = run_pointwise(p, c, nb, c, batch, nullptr, s))) return st;
    return transform(p, true, c, c, batch, glb, s);
}
