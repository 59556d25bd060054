// bc_runtime.hpp -- contexts and plans behind the C ABI.
#pragma once

#include <cstdint>
#include <list>
#include <memory>
#include <mutex>
#include <vector>

#include <cuda_runtime.h>

#include "bc_common.hpp"
#include "bc_kernels.hpp"

struct bc_plan;

// One per GPU: a stream, a device status word and a cache of plans used by
// the single-polynomial reference-op entry points.
struct bc_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    uint32_t *h_status = nullptr;  // status word: mapped page-locked host memory
    uint32_t *d_status = nullptr;  // its device address (what kernels store to)
    // Stream-ordered pool for per-call temporaries (multi-pass transforms):
    // each call allocates and frees on its own stream, so calls on several
    // streams never share or free a buffer another stream still uses.
    cudaMemPool_t pool = nullptr;
    std::mutex cache_mu;
    struct CacheEntry {
        uint32_t degree;
        uint64_t modulus, root, inv_root;
        int mode;
        std::shared_ptr<bc_plan> plan;  // callers hold a reference while they use it
    };
    std::list<CacheEntry> cache;  // most recent first
};

enum class KernelKind : int { Smem = 0, Cluster = 1, Global = 2, Scale = 3 };

struct bc_plan {
    bc_ctx *ctx = nullptr;
    uint32_t degree = 0, logn = 0, n_limbs = 0;
    int mode = BC_NTT_CYCLIC;
    bc::Word word = bc::Word::W64;
    KernelKind kind = KernelKind::Smem;
    int cluster = 1;
    std::vector<uint64_t> moduli, roots, inv_roots;
    std::vector<bc::LimbConst> limbs;
    bc::LimbConst *d_limbs = nullptr;
    bc::CoeffConst *d_coeff = nullptr;  // per-limb constants of the coefficient-wise ops
    void *d_tw_fwd = nullptr;  // forward CT table
    void *d_tw_inv = nullptr;  // inverse table (CT for cyclic, GS for negacyclic), N^-1 folded
    void *d_tw_fwd_fast = nullptr;  // the same tables in the fast kernels' layout
    void *d_tw_inv_fast = nullptr;
    // Cyclic plans whose roots are all primitive N-th roots with inv_root =
    // root^-1: the inverse as a Gentleman-Sande network (fast layout, N^-1
    // folded into its last stage), which exactly undoes the forward and so
    // lets the fused product serve cyclic plans.  Null otherwise.
    void *d_tw_gs_fast = nullptr;
    uint64_t table_bytes = 0;
};

namespace bc {

// Sets the device of `ctx` current on the calling thread.
int use_device(const bc_ctx *ctx);
// Maps a CUDA error to a status (and records the message).
int cuda_fail(cudaError_t e, const char *what);
// Host-side table entry (w, w') of limb `limb`; table 0 forward, 1 inverse.
void table_entry(const bc_plan &p, uint32_t limb, int table, uint32_t k, uint64_t *w,
                 uint64_t *wq);
// Whether a cyclic plan's roots allow the Gentleman-Sande form of its inverse
// (every root a primitive N-th root, inv_root its exact inverse).
bool cyclic_roots_primitive(const bc_plan &p);
// Builds limb constants and tables on the host (no device work).
int plan_build_host(bc_plan &p, uint32_t degree, uint32_t n_limbs, const uint64_t *moduli,
                    const uint64_t *roots, const uint64_t *inv_roots, int mode,
                    std::vector<unsigned char> *fwd, std::vector<unsigned char> *inv);
// Plan for the reference-op entry points, cached per context.  The caller's
// reference keeps the plan alive if the cache evicts it meanwhile (another
// thread filling the cache), so it is destroyed only after its last use.
int cached_plan(bc_ctx *ctx, uint32_t degree, uint64_t modulus, uint64_t root,
                uint64_t inv_root, int mode, std::shared_ptr<bc_plan> *out);
// Waits for the context stream and converts kernel status bits to errors.
int ctx_sync(bc_ctx *ctx);

int run_forward(bc_plan *p, const uint64_t *in, uint64_t *out, uint32_t batch,
                const bc_layout *layout, cudaStream_t s);
int run_inverse(bc_plan *p, const uint64_t *in, uint64_t *out, uint32_t batch,
                const bc_layout *layout, cudaStream_t s);
int run_pointwise(bc_plan *p, const uint64_t *a, const uint64_t *b, uint64_t *c,
                  uint32_t batch, const bc_layout *layout, cudaStream_t s);
int run_polymul(bc_plan *p, const uint64_t *a, const uint64_t *b, uint64_t *c,
                uint32_t batch, const bc_layout *layout, cudaStream_t s);
// Whether run_polymul would take its unfused path, which allocates, syncs
// and frees a temporary buffer (false when the arguments are invalid).
bool polymul_allocates(bc_plan *p, const uint64_t *a, const uint64_t *b, uint64_t *c,
                       uint32_t batch, const bc_layout *layout);

}  // namespace bc
