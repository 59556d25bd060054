// bc_calibrate.cu -- integer-pipe butterfly peak of this GPU, the second
// term of the NTT roofline (the slower of bytes at HBM peak and modular
// butterflies at this peak).
//
// Every thread runs Cooley-Tukey butterflies on 16 words held in registers,
// with the arithmetic the plans use for the given word size (32-bit Shoup
// with lazy [0, 2q) reduction for q < 2^31, 64-bit Shoup/Harvey for larger
// moduli), pairing words at distance 8, 4, 2, 1 as a radix-2 network does.
// No memory traffic happens between the first and the last round, so the
// rate is what the SM's issue slots and integer pipes sustain.
#include <cstdint>

#include <cuda_runtime.h>

#include "bc_common.hpp"
#include "bc_kernels.hpp"
#include "bc_runtime.hpp"

namespace bc {
namespace {

constexpr int kWords = 16;
constexpr unsigned kThreads = 256;

template <class A>
__global__ void __launch_bounds__(kThreads) k_butterfly_peak(typename A::W q, typename A::W w, typename A::W wq,
                                                             uint32_t rounds, uint64_t sentinel, uint64_t *sink) {
    using W = typename A::W;
    W v[kWords];
#pragma unroll
    for (int i = 0; i < kWords; ++i) v[i] = static_cast<W>((threadIdx.x * 2654435761u + i * 40503u) % q);
    for (uint32_t r = 0; r < rounds; ++r) {
#pragma unroll
        for (int d = kWords / 2; d >= 1; d /= 2) {
#pragma unroll
            for (int i = 0; i < kWords; ++i)
                if ((i & d) == 0) A::ct(v[i], v[i + d], w, wq, q);
        }
    }
    uint64_t acc = 0;
#pragma unroll
    for (int i = 0; i < kWords; ++i) acc ^= static_cast<uint64_t>(v[i]);
    // the results must be observable, or the rounds would be dead code: a
    // sentinel the compiler cannot know (the host passes one no result hits)
    if (acc == sentinel) sink[threadIdx.x] = acc;
}

template <class A>
int time_kernel(typename A::W q, typename A::W w, typename A::W wq, uint32_t rounds, unsigned blocks, uint64_t *sink,
                cudaStream_t s, float *ms) {
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    const uint64_t sentinel = ~0ull;  // above every word of both flavours' moduli
    k_butterfly_peak<A><<<blocks, kThreads, 0, s>>>(q, w, wq, rounds / 8, sentinel, sink);  // warm-up
    cudaEventRecord(e0, s);
    k_butterfly_peak<A><<<blocks, kThreads, 0, s>>>(q, w, wq, rounds, sentinel, sink);
    cudaEventRecord(e1, s);
    cudaError_t e = cudaEventSynchronize(e1);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaEventElapsedTime(ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    return e == cudaSuccess ? BC_OK : cuda_fail(e, "butterfly calibration");
}

}  // namespace
}  // namespace bc

using namespace bc;

extern "C" int bc_calibrate_butterflies(bc_ctx *ctx, int word_bits, double *butterflies_per_s) {
    if (!ctx || !butterflies_per_s) return fail(BC_ERR_INVALID_INPUT, "NULL argument");
    if (word_bits != 32 && word_bits != 64)
        return fail(BC_ERR_INVALID_INPUT, format("word_bits must be 32 or 64, got %d", word_bits));
    int st = use_device(ctx);
    if (st) return st;
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ctx->device);
    const unsigned blocks = static_cast<unsigned>(sms) * 8;  // 64 warps per SM
    const uint32_t rounds = word_bits == 32 ? 4096 : 1024;
    uint64_t *sink = nullptr;
    cudaError_t e = cudaMalloc(&sink, kThreads * sizeof(uint64_t));
    if (e != cudaSuccess) return cuda_fail(e, "calibration buffer");
    float ms = 0.f;
    if (word_bits == 32) {  // the largest prime below 2^31 with q = 1 mod 2^18 (N = 2^17)
        const uint32_t q = 2146959361u, w = 1234567u;
        const uint32_t wq = static_cast<uint32_t>((static_cast<uint64_t>(w) << 32) / q);
        st = time_kernel<Arith32<false>>(q, w, wq, rounds, blocks, sink, ctx->stream, &ms);
    } else {  // the largest prime below 2^60 with q = 1 mod 2^16 (N = 2^15)
        const uint64_t q = 1152921504606584833ull, w = 0x123456789ABCDull;
        const uint64_t wq = static_cast<uint64_t>((static_cast<unsigned __int128>(w) << 64) / q);
        st = time_kernel<Arith64>(q, w, wq, rounds, blocks, sink, ctx->stream, &ms);
    }
    cudaFree(sink);
    if (st) return st;
    const double butterflies = static_cast<double>(blocks) * kThreads * rounds * (kWords / 2) * 4;  // 4 levels
    *butterflies_per_s = butterflies / (ms / 1000.0);
    return BC_OK;
}
