// matvec_rows.cuh — the HBM-streaming quantized matvec for one or two
// activation vectors (batch 1 decode), block size 32.
//
// Computes y[m][n] = sum_b scale[n][b] * sum_i q[n][b][i] * x[m][32b+i] on the
// reference's native Q8_0 / Q4_0 rows (src/nn/backend.cpp:131-199 is the
// operation replaced; src/tensor/quantize.cpp:187-239 the per-row dot).
//
// One CTA per SM owns a contiguous range of rows = a contiguous byte range of
// the weight, streamed G rows per stage through a ring of nst shared-memory
// slots with 1-D bulk copies (cp.async.bulk, completion on an mbarrier, L2
// evict-first).  Stage s is computed by warp s % 16 alone, so a warp owns whole
// rows and no cross-warp reduction or CTA barrier sits on the streaming path.
// There is no producer warp: the first nst stages are issued at start, and the
// warp that finishes stage s issues stage s + nst into the slot it just read.
// Because a slot's consecutive stages belong to different warps, a warp could
// otherwise wait on a slot's barrier two phases ahead of its current phase,
// which a parity wait cannot tell from the phase before; the issuing lane
// therefore publishes the stage id it has put in the slot, and a warp waits
// for its own stage id before its parity wait.
//
// Activations are staged once per CTA in shared memory, 36 floats per 32-element
// block (4 floats of padding) so that the 16-byte reads of lanes holding
// consecutive blocks hit distinct banks.  Lane l handles blocks l, l+32, ...
// of each row; its W block is 36 B (Q8) or 18 B (Q4) read with 32-bit loads.
//
// Codes become floats with the exponent magic-number method: the code bits are
// placed in the mantissa of 2^23 and a constant is subtracted, exactly.
//  * Q8: PRMT puts the sign-flipped byte under 0x4B000000; subtract 2^23+128.
//  * Q4 FAST: a LOP3 keeps a nibble IN PLACE (bit 4k) under 0x4B000000, giving
//    2^23 + 16^k * nib; subtracting 2^23 + 8*16^k gives 16^k * q exactly, and
//    the activation was staged pre-multiplied by 16^-k (k = element % 4), so the
//    product is q*x with a single rounding, as fma(q, x, acc) would have it.
//  * Q4 EXACT: PRMT of the isolated nibble (no pre-scaling, so no underflow
//    can make a product differ from the reference's).
// FAST pairs adjacent elements in packed fp32x2 FMAs (__ffma2_rn).  EXACT uses
// scalar __fmul_rn / __fadd_rn in the reference's order: block_sum is the
// sequential chain of fl(q*x), p_b = fl(block_sum*scale) goes to a per-warp
// buffer, and one lane per row runs total = fl(total + p_b) in block order.
//
// With `pdl` set, the kernel allows the next kernel in the stream to start
// (programmatic dependent launch) and issues its weight copies before waiting
// on the previous kernel; activations are read and outputs written only after
// griddepcontrol.wait.  This overlaps one launch's ramp with the previous
// launch's tail; it requires that the immediately preceding kernel does not
// write the weight.
#pragma once

#include "common.cuh"

namespace qraf_dev {

constexpr int kRowWarps = 16;                      // warps per CTA (4 per SM sub-partition)
constexpr int kRowThreads = kRowWarps * 32;
constexpr int kRowGMax = 4;                        // rows per stage, at most

struct RowParams {
    const uint8_t* w;        // [N][row_bytes], 16-byte aligned, row_bytes % 16 == 0
    const float* x;          // [M][K]
    float* y;                // [M][N]
    uint64_t row_bytes;
    uint32_t N, K, M;        // M = activation vectors of this launch
    uint32_t nblk, nchunk;   // K / 32, ceil(nblk / 32)
    uint32_t G;              // rows per stage (1..kRowGMax)
    uint32_t nst;            // slots in the ring
    uint32_t slot_stride;    // bytes per slot (multiple of 128)
    uint32_t xs_stride;      // floats per staged activation vector = nblk * 36
    uint32_t pb_row;         // EXACT: floats per row of the per-warp partial buffer
    uint32_t rows_base, rows_extra;
    uint32_t pdl;            // 1: programmatic dependent launch protocol
};

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Wait (bounded) until the issuing lane has published stage `s` in this slot.
__device__ __forceinline__ bool wait_stage_id(volatile uint32_t* slot_stage, uint32_t s) {
    if (*slot_stage == s) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 0;; ++it) {
        __nanosleep(32);
        if (*slot_stage == s) return true;
        if ((it & 63u) == 63u && globaltimer_ns() - t0 > kWaitLimitNs) {
            raise_error(kErrWaitTimeout);
            return false;
        }
    }
}

// 32 staged activations of block b of vector v.
__device__ __forceinline__ void lds_x_block(const float* xs, uint32_t b, float4 (&xv)[8]) {
    const float4* p = reinterpret_cast<const float4*>(xs + 36u * b);
#pragma unroll
    for (int i = 0; i < 8; ++i) xv[i] = p[i];
}

// ── FAST block dots: returns the block's sum (before its scale) ──────────
__device__ __forceinline__ float q8_block_fast(const uint32_t (&wv)[9], const float4 (&xv)[8]) {
    const float2 negc = make_float2(-kMagicQ8, -kMagicQ8);
    float2 a0 = make_float2(0.0f, 0.0f), a1 = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t u = wv[1 + j] ^ 0x80808080u;
        const float2 q01 = f2_add(make_float2(magic_byte(u, 0), magic_byte(u, 1)), negc);
        const float2 q23 = f2_add(make_float2(magic_byte(u, 2), magic_byte(u, 3)), negc);
        a0 = f2_fma(q01, make_float2(xv[j].x, xv[j].y), a0);
        a1 = f2_fma(q23, make_float2(xv[j].z, xv[j].w), a1);
    }
    const float2 s = f2_add(a0, a1);
    return s.x + s.y;
}

// Q4 FAST: x was staged as x * 16^-(e % 4).  Word j holds elements 8j..8j+7;
// element e sits at bit 4*(e % 8) of the word, i.e. at bit 4*(e % 4) of the
// word (e % 8 < 4) or of the word shifted right by 16 (e % 8 >= 4).
__device__ __forceinline__ float q4_block_fast(const uint32_t (&qw)[4], const float4 (&xv)[8]) {
    const float2 c01 = make_float2(-8388616.0f, -8388736.0f);     // -(2^23 + 8), -(2^23 + 128)
    const float2 c23 = make_float2(-8390656.0f, -8421376.0f);     // -(2^23 + 2048), -(2^23 + 32768)
    float2 a0 = make_float2(0.0f, 0.0f), a1 = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t lo = qw[j], hi = qw[j] >> 16;
        const float2 q01 = f2_add(make_float2(__uint_as_float((lo & 0x000Fu) | kMagicBits),
                                              __uint_as_float((lo & 0x00F0u) | kMagicBits)), c01);
        const float2 q23 = f2_add(make_float2(__uint_as_float((lo & 0x0F00u) | kMagicBits),
                                              __uint_as_float((lo & 0xF000u) | kMagicBits)), c23);
        const float2 q45 = f2_add(make_float2(__uint_as_float((hi & 0x000Fu) | kMagicBits),
                                              __uint_as_float((hi & 0x00F0u) | kMagicBits)), c01);
        const float2 q67 = f2_add(make_float2(__uint_as_float((hi & 0x0F00u) | kMagicBits),
                                              __uint_as_float((hi & 0xF000u) | kMagicBits)), c23);
        const float4 xa = xv[2 * j], xb = xv[2 * j + 1];
        a0 = f2_fma(q01, make_float2(xa.x, xa.y), a0);
        a1 = f2_fma(q23, make_float2(xa.z, xa.w), a1);
        a0 = f2_fma(q45, make_float2(xb.x, xb.y), a0);
        a1 = f2_fma(q67, make_float2(xb.z, xb.w), a1);
    }
    const float2 s = f2_add(a0, a1);
    return s.x + s.y;
}

// ── EXACT block dots: the reference's order, scalar, never fused ─────────
__device__ __forceinline__ float q8_block_exact(const uint32_t (&wv)[9], const float4 (&xv)[8]) {
    float acc = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t u = wv[1 + j] ^ 0x80808080u;
        acc = __fadd_rn(acc, __fmul_rn(magic_byte(u, 0) - kMagicQ8, xv[j].x));
        acc = __fadd_rn(acc, __fmul_rn(magic_byte(u, 1) - kMagicQ8, xv[j].y));
        acc = __fadd_rn(acc, __fmul_rn(magic_byte(u, 2) - kMagicQ8, xv[j].z));
        acc = __fadd_rn(acc, __fmul_rn(magic_byte(u, 3) - kMagicQ8, xv[j].w));
    }
    return __fmul_rn(acc, __uint_as_float(wv[0]));
}

__device__ __forceinline__ float q4_block_exact(const uint32_t (&qw)[4], uint32_t s16, const float4 (&xv)[8]) {
    float acc = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t lo = qw[j] & 0x0F0F0F0Fu, hi = (qw[j] >> 4) & 0x0F0F0F0Fu;
        const float4 xa = xv[2 * j], xb = xv[2 * j + 1];
        acc = __fadd_rn(acc, __fmul_rn(magic_byte(lo, 0) - kMagicQ4, xa.x));
        acc = __fadd_rn(acc, __fmul_rn(magic_byte(hi, 0) - kMagicQ4, xa.y));
        acc = __fadd_rn(acc, __fmul_rn(magic_byte(lo, 1) - kMagicQ4, xa.z));
        acc = __fadd_rn(acc, __fmul_rn(magic_byte(hi, 1) - kMagicQ4, xa.w));
        acc = __fadd_rn(acc, __fmul_rn(magic_byte(lo, 2) - kMagicQ4, xb.x));
        acc = __fadd_rn(acc, __fmul_rn(magic_byte(hi, 2) - kMagicQ4, xb.y));
        acc = __fadd_rn(acc, __fmul_rn(magic_byte(lo, 3) - kMagicQ4, xb.z));
        acc = __fadd_rn(acc, __fmul_rn(magic_byte(hi, 3) - kMagicQ4, xb.w));
    }
    return __fmul_rn(acc, half_bits_to_float(s16));
}

// ── the kernel ────────────────────────────────────────────────────────────
template <uint32_t DT, bool EXACT, int MT>
__global__ void __launch_bounds__(kRowThreads, 1) qmv_rows_kernel(const RowParams p) {
    static_assert(MT == 1 || MT == 2, "one or two activation vectors per pass");
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t nst = p.nst;
    uint8_t* slots = smem;
    float* xs = reinterpret_cast<float*>(smem + static_cast<size_t>(nst) * p.slot_stride);
    float* pbuf = xs + static_cast<size_t>(p.M) * p.xs_stride;                          // EXACT only
    uint64_t* full = reinterpret_cast<uint64_t*>(
        pbuf + (EXACT ? static_cast<size_t>(kRowWarps) * p.G * p.pb_row : 0));
    volatile uint32_t* slot_stage = reinterpret_cast<volatile uint32_t*>(full + nst);

    if (blockDim.x != static_cast<uint32_t>(kRowThreads)) {
        if (threadIdx.x == 0) raise_error(kErrBadLaunch);
        return;
    }
    const uint32_t c = blockIdx.x;
    const uint32_t r0 = c * p.rows_base + min(c, p.rows_extra);
    const uint32_t nrows = p.rows_base + (c < p.rows_extra ? 1u : 0u);
    const uint32_t nstages = (nrows + p.G - 1) / p.G;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < nst; ++s) {
            mbar_init(&full[s], 1);
            slot_stage[s] = 0xFFFFFFFFu;
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (p.pdl) pdl_launch_dependents();

    // Issue one stage's rows into its slot (one lane).  Weights are read-only
    // model data, so the first stages go out before the dependency wait.
    const uint64_t pol = policy_evict_first();
    auto issue = [&](uint32_t s) {
        const uint32_t slot = s % nst;
        const uint32_t bytes = min(p.G, nrows - s * p.G) * static_cast<uint32_t>(p.row_bytes);
        mbar_arrive_expect_tx(&full[slot], bytes);
        bulk_g2s(slots + static_cast<size_t>(slot) * p.slot_stride,
                 p.w + static_cast<size_t>(r0 + s * p.G) * p.row_bytes, bytes, &full[slot], pol);
        slot_stage[slot] = s;   // the slot's barrier is now in stage s's phase
    };
    if (lane == 0)
        for (uint32_t s = warp; s < min(nst, nstages); s += kRowWarps) issue(s);

    // ── stage the activations (after the previous kernel finished) ──
    if (p.pdl) pdl_wait();
    {
        const uint32_t n4 = p.K / 4u;
        const uint32_t total = p.M * n4;
        for (uint32_t i = threadIdx.x; i < total; i += kRowWarps * 32u) {
            const uint32_t m = i / n4, e = (i % n4) * 4u;
            // L2-coherent load: under programmatic dependent launch x may have just been
            // written by the previous kernel, so no L1 copy of it may be trusted.
            float4 v = __ldcg(reinterpret_cast<const float4*>(p.x + static_cast<size_t>(m) * p.K) + (i % n4));
            if constexpr (DT == kDtypeQ4 && !EXACT) {
                // element e % 4 == 0,1,2,3 -> pre-scale by 16^0, 16^-1, 16^-2, 16^-3
                v.y *= 0.0625f;
                v.z *= 0.00390625f;
                v.w *= 0.000244140625f;
            }
            *reinterpret_cast<float4*>(xs + static_cast<size_t>(m) * p.xs_stride + 36u * (e >> 5) + (e & 31u)) = v;
        }
        __syncthreads();
    }

    for (uint32_t s = warp; s < nstages; s += kRowWarps) {
        const uint32_t slot = s % nst;
        if (!wait_stage_id(slot_stage + slot, s)) return;
        if (!mbar_wait(&full[slot], (s / nst) & 1u)) return;
        const uint32_t rows_s = min(p.G, nrows - s * p.G);
        const uint32_t row0 = r0 + s * p.G;
        const uint8_t* sb = slots + static_cast<size_t>(slot) * p.slot_stride;

        if constexpr (!EXACT) {
            float racc[kRowGMax][MT];
#pragma unroll
            for (int g = 0; g < kRowGMax; ++g)
#pragma unroll
                for (int v = 0; v < MT; ++v) racc[g][v] = 0.0f;
            for (uint32_t ch = 0; ch < p.nchunk; ++ch) {
                const uint32_t b = ch * 32u + lane;
                if (b < p.nblk) {
                    float4 xv[MT][8];
#pragma unroll
                    for (int v = 0; v < MT; ++v) lds_x_block(xs + static_cast<size_t>(v) * p.xs_stride, b, xv[v]);
                    if constexpr (DT == kDtypeQ8) {
                        uint32_t wv[kRowGMax][9];
#pragma unroll
                        for (int g = 0; g < kRowGMax; ++g)
                            if (g < static_cast<int>(rows_s)) load_q8_block(sb + static_cast<size_t>(g) * p.row_bytes, b, wv[g]);
#pragma unroll
                        for (int g = 0; g < kRowGMax; ++g) {
                            if (g < static_cast<int>(rows_s)) {
                                const float sc = __uint_as_float(wv[g][0]);
#pragma unroll
                                for (int v = 0; v < MT; ++v) racc[g][v] = fmaf(q8_block_fast(wv[g], xv[v]), sc, racc[g][v]);
                            }
                        }
                    } else {
                        uint32_t qw[kRowGMax][4], s16[kRowGMax];
#pragma unroll
                        for (int g = 0; g < kRowGMax; ++g)
                            if (g < static_cast<int>(rows_s))
                                load_q4_block(sb + static_cast<size_t>(g) * p.row_bytes, b, qw[g], s16[g]);
#pragma unroll
                        for (int g = 0; g < kRowGMax; ++g) {
                            if (g < static_cast<int>(rows_s)) {
                                const float sc = half_bits_to_float(s16[g]);
#pragma unroll
                                for (int v = 0; v < MT; ++v) racc[g][v] = fmaf(q4_block_fast(qw[g], xv[v]), sc, racc[g][v]);
                            }
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0 && s + nst < nstages) issue(s + nst);   // the slot's bytes are no longer read
#pragma unroll
            for (int g = 0; g < kRowGMax; ++g) {
                if (g < static_cast<int>(rows_s)) {
#pragma unroll
                    for (int v = 0; v < MT; ++v) {
                        const float t = warp_sum(racc[g][v]);
                        if (lane == 0) p.y[static_cast<size_t>(v) * p.N + row0 + g] = t;
                    }
                }
            }
        } else {
            float* pb = pbuf + static_cast<size_t>(warp) * p.G * p.pb_row;
            for (uint32_t m = 0; m < p.M; ++m) {
                const float* xm = xs + static_cast<size_t>(m) * p.xs_stride;
                for (uint32_t ch = 0; ch < p.nchunk; ++ch) {
                    const uint32_t b = ch * 32u + lane;
                    if (b < p.nblk) {
                        float4 xv[8];
                        lds_x_block(xm, b, xv);
                        for (uint32_t g = 0; g < rows_s; ++g) {
                            const uint8_t* row = sb + static_cast<size_t>(g) * p.row_bytes;
                            float pv;
                            if constexpr (DT == kDtypeQ8) {
                                uint32_t wv[9];
                                load_q8_block(row, b, wv);
                                pv = q8_block_exact(wv, xv);
                            } else {
                                uint32_t qw[4], s16;
                                load_q4_block(row, b, qw, s16);
                                pv = q4_block_exact(qw, s16, xv);
                            }
                            pb[static_cast<size_t>(g) * p.pb_row + b] = pv;
                        }
                    }
                }
                __syncwarp();
                if (lane < rows_s) {
                    // total = fl(total + p_b) in block order (quantize.cpp:205)
                    const float4* q4 = reinterpret_cast<const float4*>(pb + static_cast<size_t>(lane) * p.pb_row);
                    float total = 0.0f;
                    for (uint32_t i = 0; i < p.nblk / 4u; ++i) {
                        const float4 v = q4[i];
                        total = __fadd_rn(total, v.x);
                        total = __fadd_rn(total, v.y);
                        total = __fadd_rn(total, v.z);
                        total = __fadd_rn(total, v.w);
                    }
                    p.y[static_cast<size_t>(m) * p.N + row0 + lane] = total;
                }
                __syncwarp();
            }
            if (lane == 0 && s + nst < nstages) issue(s + nst);
        }
    }
}

}  // namespace qraf_dev
