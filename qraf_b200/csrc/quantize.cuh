// quantize.cuh — device quantizers and dequantizer, byte-exact with the
// reference's CPU code.
//
// quantize_q8_0 follows src/tensor/quantize.cpp:105-140 and quantize_q4_0
// :144-183, operation for operation: the block max of |x|, scale = max/127 (or
// /7) by IEEE division, inv = 1/scale by IEEE division (0 when scale is not
// positive), x*inv, the reference's clamp (std::min / std::max, whose NaN
// behaviour is kept: a NaN second argument returns the first), round half away
// from zero, and for Q4 the truncating fp16 encoding of the scale
// (src/tensor/dtype.cpp:39-59).  Bytes of a ragged last block that the
// reference never writes are written as 0, as its zero-initialised vector has.
#pragma once

#include "common.cuh"

namespace qraf_dev {

__device__ __forceinline__ float ref_min(float a, float b) { return (b < a) ? b : a; }
__device__ __forceinline__ float ref_max(float a, float b) { return (a < b) ? b : a; }

// fp32 -> fp16 bits with the reference's truncation (dtype.cpp:39-59).
__device__ __forceinline__ uint32_t f32_to_f16_trunc(float f) {
    const uint32_t bits = __float_as_uint(f);
    const uint32_t sign = (bits >> 31) & 1u;
    const int32_t e = static_cast<int32_t>((bits >> 23) & 0xFFu) - 127;
    const uint32_t m = bits & 0x7FFFFFu;
    if (e > 15) return (sign << 15) | 0x7C00u;
    if (e > -15) return (sign << 15) | (static_cast<uint32_t>(e + 15) << 10) | (m >> 13);
    return sign << 15;
}

struct QuantParams {
    const float* x;
    uint8_t* out;
    uint64_t nblocks_total;   // blocks over the whole launch
    uint64_t blocks_per_row;  // blocks per independently quantized row
    uint64_t row_elems;       // elements per row (the whole array for 1-row quantization)
    uint32_t bs, block_bytes;
};

// One thread per block.  Writes every byte of its block.
template <uint32_t DT>
__global__ void __launch_bounds__(256) quantize_kernel(const QuantParams p) {
    const uint64_t gb = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (gb >= p.nblocks_total) return;
    const uint64_t row = gb / p.blocks_per_row;
    const uint64_t b = gb % p.blocks_per_row;
    const uint64_t off = b * p.bs;
    const float* src = p.x + row * p.row_elems + off;
    const uint32_t n = static_cast<uint32_t>(min(static_cast<uint64_t>(p.bs), p.row_elems - off));
    uint8_t* dst = p.out + gb * p.block_bytes;

    float max_abs = 0.0f;
    for (uint32_t i = 0; i < n; ++i) {
        const float a = fabsf(src[i]);
        if (a > max_abs) max_abs = a;
    }
    if constexpr (DT == kDtypeQ8) {
        const float scale = __fdiv_rn(max_abs, 127.0f);
        const float inv = (scale > 0.0f) ? __fdiv_rn(1.0f, scale) : 0.0f;
        const uint32_t sb = __float_as_uint(scale);
        dst[0] = sb & 0xFFu; dst[1] = (sb >> 8) & 0xFFu; dst[2] = (sb >> 16) & 0xFFu; dst[3] = sb >> 24;
        for (uint32_t i = 0; i < p.bs; ++i) {
            int8_t q = 0;
            if (i < n) {
                float v = __fmul_rn(src[i], inv);
                v = ref_max(-127.0f, ref_min(127.0f, v));
                q = static_cast<int8_t>(roundf(v));
            }
            dst[4 + i] = static_cast<uint8_t>(q);
        }
    } else {
        const float scale = __fdiv_rn(max_abs, 7.0f);
        const float inv = (scale > 0.0f) ? __fdiv_rn(1.0f, scale) : 0.0f;
        const uint32_t h = f32_to_f16_trunc(scale);
        dst[0] = h & 0xFFu; dst[1] = (h >> 8) & 0xFFu;
        for (uint32_t i = 0; i < p.bs / 2u; ++i) {
            uint8_t byte = 0;
            if (i < n / 2u) {
                float v0 = __fmul_rn(src[2 * i], inv);
                float v1 = __fmul_rn(src[2 * i + 1], inv);
                v0 = ref_max(-8.0f, ref_min(7.0f, roundf(v0)));
                v1 = ref_max(-8.0f, ref_min(7.0f, roundf(v1)));
                const uint32_t lo = static_cast<uint32_t>(static_cast<int>(v0) + 8) & 0x0Fu;
                const uint32_t hi = static_cast<uint32_t>(static_cast<int>(v1) + 8) & 0x0Fu;
                byte = static_cast<uint8_t>(lo | (hi << 4));
            }
            dst[2 + i] = byte;
        }
    }
}

// Dequantize (src/tensor/quantize.cpp:17-51, 55-101): one thread per block;
// elements the reference never writes (past `count`, or the unpaired last
// element of an odd Q4 block) are 0, as in its zero-initialised tensor.
template <uint32_t DT>
__global__ void __launch_bounds__(256) dequantize_kernel(const uint8_t* q, float* out, uint64_t count, uint32_t bs,
                                                         uint32_t block_bytes, uint64_t nblocks) {
    const uint64_t b = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    const uint8_t* blk = q + b * block_bytes;
    const uint64_t off = b * bs;
    const uint32_t n = static_cast<uint32_t>(min(static_cast<uint64_t>(bs), count - off));
    if constexpr (DT == kDtypeQ8) {
        const float scale = __uint_as_float(ld_u32_unaligned(blk));
        for (uint32_t i = 0; i < n; ++i) out[off + i] = __fmul_rn(static_cast<float>(static_cast<int8_t>(blk[4 + i])), scale);
    } else {
        const float scale = half_bits_to_float(static_cast<uint32_t>(blk[0]) | (static_cast<uint32_t>(blk[1]) << 8));
        for (uint32_t i = 0; i < n / 2u; ++i) {
            const uint8_t v = blk[2 + i];
            out[off + 2 * i] = __fmul_rn(static_cast<float>(static_cast<int>(v & 0x0Fu) - 8), scale);
            out[off + 2 * i + 1] = __fmul_rn(static_cast<float>(static_cast<int>((v >> 4) & 0x0Fu) - 8), scale);
        }
        if (n & 1u) out[off + n - 1] = 0.0f;
    }
}

}  // namespace qraf_dev
