// matvec_generic.cuh — quantized matvec for any block size, any K, any alignment.
//
// One warp per (row, activation vector); lanes take blocks lane, lane+32, ...
// Bytes are read individually, so nothing about the row's alignment is
// assumed.  This covers what the streaming kernel does not: block sizes other
// than 32, a ragged last block (K not a multiple of the block size, where the
// reference still advances a full block, src/tensor/quantize.cpp:199-206 and
// :224-235), odd Q4 block sizes (the unpaired last element is not stored and
// contributes nothing), and unaligned pointers.
//
// EXACT keeps the reference's order: each lane forms p_b = fl(block_sum*scale)
// with the sequential fl(q*x) chain, the warp stages 32 consecutive p_b in
// shared memory and lane 0 adds them to the running total in block order.
// With WRITE_PARTIALS the p_b are stored instead ([row][block]), which exposes
// the per-block partial sums for bit-exact checking.
#pragma once

#include "common.cuh"

namespace qraf_dev {

struct GenericParams {
    const uint8_t* w;
    const float* x;     // [M][K]
    float* y;           // [M][N]            (or partials [N][nblk])
    uint64_t row_bytes;
    uint32_t N, K, M, bs, nblk, block_bytes;
};

template <uint32_t DT, bool EXACT>
__device__ __forceinline__ float generic_block(const uint8_t* blk, const float* x, uint32_t n) {
    float acc = 0.0f;
    float scale;
    if constexpr (DT == kDtypeQ8) {
        scale = __uint_as_float(ld_u32_unaligned(blk));
        const int8_t* q = reinterpret_cast<const int8_t*>(blk + 4);
        for (uint32_t i = 0; i < n; ++i) {
            const float qv = static_cast<float>(q[i]);
            acc = EXACT ? __fadd_rn(acc, __fmul_rn(qv, x[i])) : fmaf(qv, x[i], acc);
        }
    } else {
        scale = half_bits_to_float(static_cast<uint32_t>(blk[0]) | (static_cast<uint32_t>(blk[1]) << 8));
        const uint8_t* q = blk + 2;
        for (uint32_t i = 0; i < n / 2u; ++i) {
            const float lo = static_cast<float>(static_cast<int>(q[i] & 0x0Fu) - 8);
            const float hi = static_cast<float>(static_cast<int>((q[i] >> 4) & 0x0Fu) - 8);
            if (EXACT) {
                acc = __fadd_rn(acc, __fmul_rn(lo, x[2 * i]));
                acc = __fadd_rn(acc, __fmul_rn(hi, x[2 * i + 1]));
            } else {
                acc = fmaf(lo, x[2 * i], acc);
                acc = fmaf(hi, x[2 * i + 1], acc);
            }
        }
    }
    return __fmul_rn(acc, scale);
}

template <uint32_t DT, bool EXACT, bool WRITE_PARTIALS>
__global__ void __launch_bounds__(256) qmv_generic_kernel(const GenericParams p) {
    __shared__ float stage[8][33];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint64_t task = static_cast<uint64_t>(blockIdx.x) * 8u + warp;
    const uint64_t ntasks = static_cast<uint64_t>(p.N) * (WRITE_PARTIALS ? 1u : p.M);
    if (task >= ntasks) return;
    const uint32_t row = static_cast<uint32_t>(task % p.N);
    const uint32_t m = static_cast<uint32_t>(task / p.N);
    const uint8_t* wrow = p.w + static_cast<size_t>(row) * p.row_bytes;
    const float* xrow = p.x + static_cast<size_t>(m) * p.K;

    float total = 0.0f;   // EXACT: running in-order chain (lane 0);  FAST: lane partial
    for (uint32_t b0 = 0; b0 < p.nblk; b0 += 32u) {
        const uint32_t b = b0 + lane;
        float pv = 0.0f;
        if (b < p.nblk) {
            const uint32_t off = b * p.bs;
            const uint32_t n = min(p.bs, p.K - off);
            pv = generic_block<DT, EXACT>(wrow + static_cast<size_t>(b) * p.block_bytes, xrow + off, n);
            if constexpr (WRITE_PARTIALS) p.y[static_cast<size_t>(row) * p.nblk + b] = pv;
        }
        if constexpr (EXACT && !WRITE_PARTIALS) {
            stage[warp][lane] = pv;
            __syncwarp();
            if (lane == 0) {
                const uint32_t cnt = min(32u, p.nblk - b0);
                for (uint32_t j = 0; j < cnt; ++j) total = __fadd_rn(total, stage[warp][j]);
            }
            __syncwarp();
        } else {
            total += pv;
        }
    }
    if constexpr (!WRITE_PARTIALS) {
        if constexpr (!EXACT) total = warp_sum(total);
        if (lane == 0) p.y[static_cast<size_t>(m) * p.N + row] = total;
    }
}

}  // namespace qraf_dev
