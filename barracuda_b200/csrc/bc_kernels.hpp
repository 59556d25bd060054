// bc_kernels.hpp -- host-side launch interface of the CUDA kernels.
#pragma once

#include <cstdint>

#include <cuda_runtime.h>

#include "bc_arith.cuh"

namespace bc {

// Flags kernels write into the context's status word.  The word lives in
// mapped, page-locked host memory: a kernel that finds a bad input stores its
// flag with a plain store (no device atomics to host memory), and the host
// reads the word after waiting for the stream, with no copy.  Each kernel
// only ever stores the same flag value, so plain stores cannot lose a flag.
enum : uint32_t {
    kStatusInputRange = 1u,  // a coefficient >= 2^32 reached a 32-bit-word plan
    kStatusWaitTimeout = 2u,  // a bounded wait on an asynchronous copy ran out
};

#ifdef __CUDACC__
__device__ __forceinline__ void store_status(uint32_t *status, uint32_t flag) {
    *reinterpret_cast<volatile uint32_t *>(status) = flag;
}
#endif

// Maps a CUDA error to a status and records the message (bc_runtime.cpp).
int cuda_fail(cudaError_t e, const char *what);

// Cluster scheduling policy of every cluster launch: load balancing of a
// cluster's CTAs over the SMs (cudaClusterSchedulingPolicyLoadBalancing).
// Measured on B200 at N = 2^16 (config 3): +2.8% against the default policy,
// which spreads them.  BARRACUDA_CLUSTER_POLICY=0|1|2 overrides (default /
// spread / load balancing); read once per process.
int cluster_policy();

// Arithmetic flavour of a plan (see bc_arith.cuh).
enum class Word : int { W32Lazy4 = 0, W32Lazy2 = 1, W64 = 2 };

// Pointwise step of the fused transforms (k_ntt_mul_fast): C = NTT(A) op B^
// or C = INTT(A^ op B^), exact mod q.
enum FuseOp : uint32_t { kFuseMul = 0, kFuseAdd = 1, kFuseSub = 2 };

// Arguments common to the transform kernels.  Strides are in u64 elements.
struct KArgs {
    const uint64_t *in;
    const uint64_t *in2;  // second operand (pointwise, polymul)
    uint64_t *out;
    int64_t limb_stride;
    int64_t poly_stride;
    uint32_t batch;
    uint32_t n_limbs;
    uint32_t logn;
    uint32_t op;          // pointwise step of the fused transforms (FuseOp)
    const void *tw;      // table used by the (first) transform, N entries per limb
    const void *tw2;     // table of the second transform (polymul inverse)
    const LimbConst *limbs;
    uint32_t *status;    // device status word
};

// One polynomial per CTA, whole polynomial in shared memory, one stage per
// barrier.  gs = false: Cooley-Tukey, natural order in, natural order out
// (bit-reversal applied at the store).  gs = true: Gentleman-Sande, input
// permuted at the load.  scale_last folds N^-1 into the last stage.
int launch_ntt_smem(Word w, bool gs, bool scale_last, const KArgs &a, cudaStream_t s);
// Shared-memory budget of launch_ntt_smem: largest log2 N it accepts.
uint32_t smem_max_logn(Word w);

// Register / shared-memory / cluster kernels (bc_kernels_fast.cu): one HBM
// round trip per transform.  Inputs and outputs must be 16-byte aligned
// with even strides (every polynomial starts on a 16-byte boundary).
bool fast_supported(Word w, uint32_t logn);
int fast_cluster_size(Word w, uint32_t logn);
int launch_ntt_fast(Word w, bool gs, bool scale_last, const KArgs &a, cudaStream_t s);
// Schedule variant the fast kernel uses for a direction, and the position
// of natural twiddle-table entry knat (= m + i) in that variant's table,
// which stores each stage's twiddles transposed per pass (pair = 2 for
// 8-byte entries, 1 for 16-byte entries).
int fast_variant_for(Word w, uint32_t logn, bool inverse);
// Negacyclic transform fused with a pointwise product on the fast schedules
// (a.in = A, a.in2 = B^, a.out = C, a.tw = that direction's fast table):
// inverse = false: C = NTT(A) * B^; inverse = true: C = INTT(A * B^).
int launch_ntt_mul_fast(Word w, bool inverse, const KArgs &a, cudaStream_t s);
// Fused negacyclic polymul on the fast schedules: a.in = A, a.in2 = NTT(B)
// in natural order (may alias a.out), a.out = C, a.tw / a.tw2 = the fast
// forward / inverse tables.  Needs the same variant in both directions.
int launch_polymul_fast(Word w, const KArgs &a, cudaStream_t s);
uint64_t fast_table_index(uint32_t L, int V, uint64_t knat, int pair);

// Stage-per-launch global-memory path for any N through a compact scratch
// buffer of n_limbs * batch * N words of the plan's width (natural tables):
// the fallback of cluster plans whose buffers the fast kernels cannot take.
int launch_ntt_global(Word w, bool gs, bool scale_last, const KArgs &a, void *scratch,
                      cudaStream_t s);

// Two- or three-pass transform of plans above the cluster kernels
// (bc_kernels_multipass.cu), 2^18 <= N <= 2^24, any layout, through the same
// kind of scratch buffer.  Its tables store the stages below the TOP pass
// permuted: natural entry knat sits at multipass_table_index(L, top_lo, knat),
// top_lo = multipass_top_lo(w, L).
bool multipass_supported(Word w, uint32_t logn);
uint32_t multipass_top_lo(Word w, uint32_t logn);
uint64_t multipass_table_index(uint32_t L, uint32_t top_lo, uint64_t knat);
int launch_ntt_multipass(Word w, bool gs, bool scale_last, const KArgs &a, void *scratch,
                         cudaStream_t s);

// C = A * B mod q per coefficient (exact; inputs < 2^32 for 32-bit words).
int launch_pointwise(Word w, const KArgs &a, cudaStream_t s);
// Reference behaviour for modulus 0 (fhe_pointwise_mul.wgsl reduce64 with
// q = 0 leaves the low 32 bits of the product): C = (A * B) mod 2^32.
int launch_mul_lo32(const KArgs &a, cudaStream_t s);
// Fused polymul, one polynomial pair per CTA in shared memory.
// cyclic: CT(a), CT(b), product, permute, CT(inverse table) with N^-1 folded.
// negacyclic: CT(a), CT(b), product, GS(inverse table) with N^-1 folded.
int launch_polymul_smem(Word w, bool cyclic, const KArgs &a, cudaStream_t s);
uint32_t polymul_smem_max_logn(Word w);
// Multiplies every coefficient by N^-1 (degree-1 inverse transform).
int launch_scale(Word w, const KArgs &a, cudaStream_t s);

// Coefficient-wise ops (FhePolyAdd / FhePolySub / FhePolyMul) on u64 words
// of any value, with one modulus per limb.
struct CoeffConst {
    uint64_t q;
    uint64_t m;   // floor((2^64 - 1) / q): quotient estimate for any u64
    uint64_t mu;  // floor(2^(2k) / q), k = bit length of q (products for 2^32 <= q < 2^62)
    uint32_t k;
    uint32_t pad;
};
CoeffConst coeff_const(uint64_t q);  // q != 0
// Add and Sub follow the reference shaders (exact for inputs below q); the
// Exact forms reduce both inputs first and are exact for any u64 (the
// two-launch path of the fused transform-and-add/sub).
enum CoeffOp : int { kCoeffAdd = 0, kCoeffSub = 1, kCoeffMul = 2, kCoeffAddExact = 3, kCoeffSubExact = 4 };
// C = A op B for a.batch polynomials of n coefficients per limb (layout
// strides in `a`); `consts` holds one CoeffConst per limb on the device, or
// is NULL and `single` serves every limb.
int launch_coeff_op(int op, const KArgs &a, uint64_t n, const CoeffConst *consts,
                    const CoeffConst &single, cudaStream_t s, bool flag_wide_words = false);

int launch_fill_uniform(const KArgs &a, uint64_t seed, uint64_t first_poly,
                        uint64_t total_polys, cudaStream_t s);
int launch_digest(const uint64_t *in, size_t count, uint64_t first, uint64_t *out, cudaStream_t s);

// ---- automorphisms, modulus switching, digit decomposition (bc_kernels_rns.cu) ----
// X -> X^galois (galois odd) on a.batch polynomials of each of a.n_limbs
// limbs: out[j] = in[t] if t < N, else q - in[t - N] (0 stays 0), where
// t = j galois^-1 mod 2N; the modulus of limb l is consts[l].q, or single_q
// when consts is NULL.  a.in and a.out must not overlap.
int launch_automorphism(const KArgs &a, uint32_t galois, const CoeffConst *consts, uint64_t single_q,
                        cudaStream_t s);
// Inverse of an odd g modulo 2^logm (logm <= 32).
uint32_t odd_inverse_pow2(uint32_t g, uint32_t logm);
// Constants of round(c q_new / q_old) mod q_new: m_old = floor(2^64 / q_old),
// p_shoup = floor(q_new 2^64 / q_old); both 0 when q_new == 0.
struct ModSwitchConst {
    uint64_t q_old, q_new, m_old, p_shoup;
};
ModSwitchConst modswitch_const(uint64_t q_old, uint64_t q_new);  // q_new < q_old
int launch_modulus_switch(const uint64_t *in, uint64_t *out, size_t count, const ModSwitchConst &c,
                          cudaStream_t s);
// out[l * count + i] = digit l (base `base`, 2 <= base <= 2^24) of in[i], l < levels.
int launch_decompose(const uint64_t *in, uint64_t *out, size_t count, uint32_t base, uint32_t levels,
                     cudaStream_t s);

}  // namespace bc
