// common.cuh — shared device helpers for the qraf_b200 kernels (sm_100a).
//
// Block formats consumed everywhere (the reference's on-disk layout,
// src/tensor/quantize.cpp:14-51, unchanged):
//   Q8_0 block = [f32 scale][bs x int8]          (4 + bs bytes)
//   Q4_0 block = [f16 scale][bs/2 x u8]           (2 + bs/2 bytes), byte i holds
//                element 2i in its low nibble and 2i+1 in its high nibble,
//                each biased by +8.
// A weight is [N rows][ceil(K/bs) blocks], rows back to back.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include "../../include/qraf_cuda.h"

namespace qraf_dev {

constexpr uint32_t kDtypeQ8 = QRAF_DTYPE_Q8_0;
constexpr uint32_t kDtypeQ4 = QRAF_DTYPE_Q4_0;

// Bit-or'ed into the per-device status word by kernels that give up.
constexpr uint32_t kErrWaitTimeout = 1u;    // an mbarrier / flag wait ran out of time
constexpr uint32_t kErrBadLaunch   = 2u;    // a kernel found its launch arguments inconsistent

// Per-device status word (each device that loads the module has its own copy).
// The library is one translation unit (capi.cu includes every kernel header),
// so the word is defined here.
__device__ uint32_t g_status = 0;

__device__ __forceinline__ void raise_error(uint32_t bits) { atomicOr(&g_status, bits); }

// ── shared-memory addresses, mbarriers, bulk copies ──────────────────────
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Wait for an mbarrier phase with a time limit.  Returns false (and raises
// kErrWaitTimeout) when the phase has not completed within `limit_ns`; the
// caller then stops its work and returns, so a lost arrival can never hang
// the GPU.
constexpr uint64_t kWaitLimitNs = 1000000000ull;   // 1 s

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 0;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 63u && globaltimer_ns() - t0 > kWaitLimitNs) {
            raise_error(kErrWaitTimeout);
            return false;
        }
    }
}

// One-dimensional bulk copy global -> shared, completing on `bar`.
// src, dst and bytes must all be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_u32(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// L2 policy for data many CTAs read (activations).
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// L2 policy for data read exactly once (streamed weights).
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Programmatic dependent launch: wait for the previous grid in the stream to
// complete (its memory visible), and let the next grid start its prologue.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Copy n floats between pinned host memory (mapped into the device's address
// space) and device memory with the SMs: for the few kilobytes of one host
// call's x or y this takes a fraction of a copy engine's latency.  Reads of
// host memory skip the caches (ld.global.cv), writes to it go straight through
// (st.global.wt).  The next kernel in the stream may launch at once; a kernel
// launched as its programmatic dependent waits for this grid before it reads dst.
// The device-to-host copy is itself launched as a programmatic dependent of the
// matvec before it (so it waits here, before reading src); a wait without such
// a launch returns at once.
// With `status_out` set (device-to-host only), one thread also takes the
// device's status word (reading and clearing it) and stores it there, so that
// the host learns of an expired wait in the kernels before it, with no extra
// copy.
template <bool FROM_HOST>
__global__ void __launch_bounds__(256) host_copy_kernel(const float* __restrict__ src, float* __restrict__ dst,
                                                        size_t n, uint32_t* status_out) {
    pdl_launch_dependents();
    if constexpr (!FROM_HOST) {
        pdl_wait();
        if (status_out && blockIdx.x == 0 && threadIdx.x == 0) __stwt(status_out, atomicExch(&g_status, 0u));
    }
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    const size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const size_t n4 = n >> 2;   // src and dst are 16-byte aligned
    const float4* s4 = reinterpret_cast<const float4*>(src);
    float4* d4 = reinterpret_cast<float4*>(dst);
    for (size_t i = t; i < n4; i += stride) {
        if constexpr (FROM_HOST) d4[i] = __ldcv(s4 + i);
        else __stwt(d4 + i, s4[i]);
    }
    for (size_t i = 4 * n4 + t; i < n; i += stride) {
        if constexpr (FROM_HOST) dst[i] = __ldcv(src + i);
        else __stwt(dst + i, src[i]);
    }
}

// ── packed fp32x2 arithmetic (sm_100a), IEEE round-to-nearest, no ftz ────
// CUDA's float2 intrinsics.  Used where rounding order is free (FAST mode):
// a packed multiply followed by a packed add was measured to round like a
// fused multiply-add on sm_100a, so EXACT code uses the scalar __fmul_rn /
// __fadd_rn forms instead.
__device__ __forceinline__ float2 f2_add(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 f2_mul(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 f2_fma(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// ── integer -> float without the conversion unit ──────────────────────────
// A byte u placed in the low mantissa bits of 2^23 gives the float 2^23 + u
// exactly; subtracting a constant then yields small integers exactly.
constexpr uint32_t kMagicBits = 0x4B000000u;          // 2^23
constexpr float kMagicQ8 = 8388736.0f;                // 2^23 + 128  (int8 stored with its sign bit flipped)
constexpr float kMagicQ4 = 8388616.0f;                // 2^23 + 8    (nibble bias of Q4_0)

// Selector for __byte_perm(v, kMagicBits, sel): byte t of v into byte 0,
// zero bytes 1-2, 0x4B into byte 3.
__device__ __forceinline__ constexpr uint32_t magic_sel(int t) { return 0x7440u | static_cast<uint32_t>(t); }

__device__ __forceinline__ float magic_byte(uint32_t v, int t) {
    return __int_as_float(static_cast<int>(__byte_perm(v, kMagicBits, magic_sel(t))));
}

// fp16 bits -> fp32, exact for every finite value, subnormals and infinities
// (the reference's decoder, src/tensor/dtype.cpp:9-37, is exact too).
__device__ __forceinline__ float half_bits_to_float(uint32_t h16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(h16 & 0xFFFFu)));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

// ── block loaders (shared memory -> registers) ────────────────────────────
// Q8: 9 words; word 0 = fp32 scale, words 1..8 = 32 int8 codes.
__device__ __forceinline__ void load_q8_block(const uint8_t* row, uint32_t b, uint32_t (&wv)[9]) {
    const uint32_t* p = reinterpret_cast<const uint32_t*>(row + 36u * b);
#pragma unroll
    for (int i = 0; i < 9; ++i) wv[i] = p[i];
}

// Q4: the 18-byte block starts on a 4-byte boundary for even b and 2 bytes
// past one for odd b.  Read the 5 aligned words covering it and funnel-shift
// the codes into 4 words; `scale16` gets the fp16 scale bits.
__device__ __forceinline__ void load_q4_block(const uint8_t* row, uint32_t b, uint32_t (&qw)[4], uint32_t& scale16) {
    const uint32_t* p = reinterpret_cast<const uint32_t*>(row) + ((9u * b) >> 1);
    uint32_t w[5];
#pragma unroll
    for (int i = 0; i < 5; ++i) w[i] = p[i];
    const uint32_t sh = (b & 1u) ? 32u : 16u;
#pragma unroll
    for (int j = 0; j < 4; ++j) qw[j] = __funnelshift_rc(w[j], w[j + 1], sh);
    scale16 = __funnelshift_rc(w[0], w[1], sh - 16u) & 0xFFFFu;
}

__device__ __forceinline__ uint32_t ld_u32_unaligned(const uint8_t* p) {
    return static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8) | (static_cast<uint32_t>(p[2]) << 16) |
           (static_cast<uint32_t>(p[3]) << 24);
}

}  // namespace qraf_dev
