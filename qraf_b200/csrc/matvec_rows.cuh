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
constexpr int kMaxWorld = 8;                       // GPUs in a row-sharded group, at most
constexpr int kMaxSeg = 4;                         // weights of one multi-weight launch, at most

struct RowParams {
    const uint8_t* w;        // [N][row_bytes], 16-byte aligned, row_bytes % 16 == 0
    const float* x;          // [M][K]
    float* y;                // [M][N]
    uint64_t row_bytes;
    uint32_t N, K, M;        // M = activation vectors of this launch
    uint32_t nblk;           // K / 32
    uint32_t G;              // rows per stage (1..kRowGMax)
    // A stage is G rows x one piece of K: pieces of `piece_blocks` blocks
    // (npieces per row; the last may be shorter; EXACT uses whole rows).  With
    // several pieces, each stage leaves its G partial sums in shared memory and
    // the rows are summed piece by piece, in order, at the end.
    uint32_t piece_blocks, npieces, piece_bytes;
    uint32_t part_rows;      // rows per CTA the partial-sum buffer is sized for
    uint32_t nst;            // slots in the ring
    uint32_t slot_stride;    // bytes per slot (multiple of 128)
    uint32_t xs_stride;      // bytes per staged activation vector: nblk * 144 (EXACT), nblk * kLimbRec (FAST)
    uint32_t pb_row;         // EXACT: floats per row of the per-warp partial buffer
    uint32_t rows_base, rows_extra;   // rows per CTA in units of row_unit rows: the first rows_extra CTAs take one more
    uint32_t row_unit;       // 1, or 2 for paired (SwiGLU) rows
    uint32_t pdl;            // 1: programmatic dependent launch protocol
    const uint8_t* xrec;     // FAST: limb records built by limb_prep_kernel ([M][nblk] x kLimbRec), or null
    uint32_t early;          // ring stages issued before the dependency wait; the rest of the first lap after
                             // the activations are staged (their loads queue behind the SM's copies in flight)
    // Several weights of one input in one launch (nseg >= 2): virtual rows
    // [seg_row0[i], seg_row0[i+1]) are the rows of weight i (seg_w[i]), whose
    // outputs go to seg_y[i] ([M][rows of weight i]); same cols, dtype and
    // row_bytes for all.  nseg <= 1: the one weight w and output y.
    uint32_t nseg;
    const uint8_t* seg_w[kMaxSeg];
    float* seg_y[kMaxSeg];
    uint32_t seg_row0[kMaxSeg + 1];
    // SwiGLU pairs (swiglu = 1, FAST, two rows per stage): virtual row 2i is row i
    // of the gate weight seg_w[0], 2i + 1 row i of the up weight seg_w[1]; the
    // stage that holds both writes silu(gate) * up (the reference's
    // x / (1 + exp(-x)), then the product: src/nn/ops.cpp:218-221,
    // src/nn/attention.cpp:172-179) to seg_y[0][v][i] ([M][N / 2]).
    uint32_t swiglu;
    // Fusions around the projection (null: none).  norm_w: x is replaced by
    // RMSNorm(x) = x * (1 / sqrt(mean(x^2) + norm_eps)) * norm_w per vector
    // (src/nn/ops.cpp:107-118; FAST only: the sum of squares is taken in fp64 by
    // the whole CTA).  seg_b[i]: a bias added to weight i's outputs, fl(y + b)
    // (src/nn/attention.cpp:100-102).
    const float* norm_w;
    float norm_eps;
    const float* seg_b[kMaxSeg];
    // accumulate = 1 (one weight, unsharded): y = fl(W x + y), the residual add of
    // a projection whose output joins the residual stream (src/nn/transformer.cpp:593,
    // :601); each element is read and written by the one thread that stores it.
    uint32_t accumulate;
    // Row-sharded launch (world > 0): this GPU computes rows [row_off, row_off + N)
    // of a y with y_ld rows in all (the ranks' row ranges partition them).  Each
    // output element goes into this rank's y and, as one 8-byte word (call number
    // << 32 | value bits), into every peer's receive array at the element's index:
    // plain stores over NVLink and no fence, since an aligned 8-byte store is seen
    // whole or not at all.  At the end every CTA copies its share of the other
    // ranks' rows from this rank's receive array into y, polling (bounded) until
    // each word carries this call's number.  Calls are numbered on the device
    // (*seq), so a captured and replayed sequence of calls stays in step.
    float* y_full;                                // this rank's y, [M_call][y_ld] (all vectors of the host call)
    uint32_t v_off;                               // this launch's first vector within the host call
    unsigned long long* peer_ll[kMaxWorld];       // rank r's receive array: two halves of ll_cap words (call parity)
    unsigned long long* local_ll;                 // this rank's receive array
    uint64_t ll_cap;
    uint32_t* cta_counter;                        // CTAs of this launch that have finished
    uint32_t* seq;                                // calls of this comm completed on this rank
    uint32_t world, rank, y_ld, row_off;
};


__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* a, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(a), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* a) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
    return v;
}

// The segment (weight) that virtual row `row` belongs to (multi-weight launches).
__device__ __forceinline__ uint32_t seg_of(const RowParams& p, uint32_t row) {
    uint32_t i = 0;
#pragma unroll
    for (int j = 1; j < kMaxSeg; ++j)
        if (static_cast<uint32_t>(j) < p.nseg && row >= p.seg_row0[j]) i = static_cast<uint32_t>(j);
    return i;
}

// First byte of virtual row `row` in global memory.
__device__ __forceinline__ const uint8_t* row_src(const RowParams& p, uint32_t row) {
    if (p.swiglu) return p.seg_w[row & 1u] + static_cast<size_t>(row >> 1) * p.row_bytes;
    if (p.nseg <= 1) return p.w + static_cast<size_t>(row) * p.row_bytes;
    const uint32_t i = seg_of(p, row);
    return p.seg_w[i] + static_cast<size_t>(row - p.seg_row0[i]) * p.row_bytes;
}

// Row-sharded store of output element (vector v of the launch, local row `row`)
// into this rank's y and, as a (call, value) word, every peer's receive array.
// P: the launch's parameters (RowParams or the tensor-core tile's TcParams, which
// carry the same sharding fields).
template <class P>
__device__ __forceinline__ void sharded_store(const P& p, uint32_t call, uint32_t v, uint32_t row, float t) {
    const size_t idx = static_cast<size_t>(v + p.v_off) * p.y_ld + p.row_off + row;
    p.y_full[idx] = t;
    const unsigned long long word = (static_cast<unsigned long long>(call) << 32) | __float_as_uint(t);
    const size_t off = static_cast<size_t>(call & 1u) * p.ll_cap + idx;
#pragma unroll
    for (int r = 0; r < kMaxWorld; ++r)
        if (r < static_cast<int>(p.world) && r != static_cast<int>(p.rank)) st_relaxed_sys_u64(p.peer_ll[r] + off, word);
}

// One output element: into y (or its weight's y), or (row-sharded) into this
// rank's y and every peer's receive array.
__device__ __forceinline__ void store_out(const RowParams& p, uint32_t call, uint32_t v, uint32_t row, float t) {
    if (p.world == 0) {
        if (p.nseg <= 1) {
            if (p.seg_b[0]) t = __fadd_rn(t, p.seg_b[0][row]);
            float* dst = p.y + static_cast<size_t>(v) * p.N + row;
            if (p.accumulate) t = __fadd_rn(t, *dst);
            *dst = t;
        } else {
            const uint32_t i = seg_of(p, row);
            const uint32_t r = row - p.seg_row0[i];
            if (p.seg_b[i]) t = __fadd_rn(t, p.seg_b[i][r]);
            p.seg_y[i][static_cast<size_t>(v) * (p.seg_row0[i + 1] - p.seg_row0[i]) + r] = t;
        }
        return;
    }
    sharded_store(p, call, v, row, t);
}

// SwiGLU output of the pair (gate, up) = virtual rows (2i, 2i + 1).
__device__ __forceinline__ void store_swiglu(const RowParams& p, uint32_t v, uint32_t pair, float g, float u) {
    if (p.seg_b[0]) g = __fadd_rn(g, p.seg_b[0][pair]);
    if (p.seg_b[1]) u = __fadd_rn(u, p.seg_b[1][pair]);
    const float act = g / (1.0f + expf(-g));
    p.seg_y[0][static_cast<size_t>(v) * (p.N >> 1) + pair] = act * u;
}

// h = silu(h) * u, element by element (the SwiGLU entry's unfused path).
__global__ void __launch_bounds__(256) swiglu_apply_kernel(float* __restrict__ h, const float* __restrict__ u,
                                                           size_t n) {
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const float g = h[i];
        h[i] = (g / (1.0f + expf(-g))) * u[i];
    }
}

// Row-sharded completion, by every thread of every CTA: copy the other ranks'
// rows of this call from the receive array into y (bounded polling), then the
// last CTA to finish records the call as completed.  A peer cannot overwrite a
// half of the receive array before this rank has finished reading it: it
// writes call c + 2 only after finishing call c + 1, which needs this rank's
// rows of c + 1, which this rank computes only after this launch (call c)
// has completed.  P as for sharded_store; p.M vectors, p.N local rows.
template <class P>
__device__ __forceinline__ void sharded_gather(const P& p, uint32_t call) {
    // this launch's vectors [v_off, v_off + M) of the host call
    const size_t base = static_cast<size_t>(p.v_off) * p.y_ld;
    const size_t total = static_cast<size_t>(p.M) * p.y_ld;
    const unsigned long long* ll = p.local_ll + static_cast<size_t>(call & 1u) * p.ll_cap + base;
    float* yf = p.y_full + base;
    const uint64_t t0 = globaltimer_ns();
    bool ok = true;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; ok && i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const uint32_t row = static_cast<uint32_t>(i % p.y_ld);
        if (row - p.row_off < p.N) continue;   // this rank's own row, stored directly
        unsigned long long w = ld_relaxed_sys_u64(ll + i);
        for (uint32_t it = 0; static_cast<uint32_t>(w >> 32) != call; ++it) {
            if ((it & 31u) == 31u && globaltimer_ns() - t0 > kWaitLimitNs) {
                raise_error(kErrWaitTimeout);
                ok = false;
                break;
            }
            w = ld_relaxed_sys_u64(ll + i);
        }
        if (ok) yf[i] = __uint_as_float(static_cast<uint32_t>(w));
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint32_t done = atomicAdd(p.cta_counter, 1u);
        if (done == gridDim.x - 1u) {
            *p.cta_counter = 0u;   // ready for the next launch
            *p.seq = call;         // read by the next launch after this grid has completed
        }
    }
}

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

// ── FAST: activations as integer limbs, codes used as they are ───────────
// Per 32-element block b of an activation vector, with e_b such that
// max |x| (1 + 2^-8) < 2^e_b:  X_i = rint(x_i * 2^(30 - e_b)), |X_i| < 2^30, and
// X_i = L0*2^24 + L1*2^16 + L2*2^8 + L3 with balanced signed digits -128 <= L_j <= 127.
// Then sum_i q_i x_i ~= 2^(e_b - 30) * sum_j 2^(8(3-j)) * D_j,  D_j = sum_i q_i L_ji,
// where every D_j is an exact int32 (dp4a), so the per-block partial sums are
// integers independent of summation order; the only roundings are X_i (half a
// unit of 2^(e_b - 30), i.e. 2^-31 of the block maximum) and the fp32 combination.
// The digits are not extracted one by one: for |X| < 2^30 the bytes of
// U = X + 0x80808080 are the digits plus 128 (the added 128s absorb every
// borrow), so U ^ 0x80808080 holds the four signed digits, least significant in
// byte 0, and a 4 x 4 byte transpose (PRMT) turns four elements' U into one word
// per digit plane.
// Record of one block in shared memory (kLimbRec bytes): limb plane j at
// bytes [32j, 32j+32), c_b = 2^(e_b - 30) at 128, the plane sums S_j (int32) at
// 144..159 (Q4 only), padding to an odd number of 16-byte units so that lanes
// reading consecutive blocks hit distinct banks.
// Q4 stores the elements of each group of 8 in the order 0,2,4,6,1,3,5,7 so
// that the low and high nibbles of a code word line up with one limb word.
constexpr uint32_t kLimbRec = 176;

struct LimbBlock {
    uint32_t L[4][8];   // limb words, plane j, 4 elements per word
};

__device__ __forceinline__ void lds_limbs(const uint8_t* rec, LimbBlock& lb) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint4 a = *reinterpret_cast<const uint4*>(rec + 32 * j);
        const uint4 b = *reinterpret_cast<const uint4*>(rec + 32 * j + 16);
        lb.L[j][0] = a.x; lb.L[j][1] = a.y; lb.L[j][2] = a.z; lb.L[j][3] = a.w;
        lb.L[j][4] = b.x; lb.L[j][5] = b.y; lb.L[j][6] = b.z; lb.L[j][7] = b.w;
    }
}

// sum_j 2^(8(3-j)) D_j as fp32 (|D_j| < 2^20, so D0*256 + D1 and D2*256 + D3 are exact int32).
__device__ __forceinline__ float combine_limbs(int d0, int d1, int d2, int d3) {
    return fmaf(__int2float_rn(d0 * 256 + d1), 65536.0f, __int2float_rn(d2 * 256 + d3));
}

// D_j = sum_i q_i L_j,i for one block: exact int32 dot products (dp4a).
__device__ __forceinline__ void q8_block_dsums(const uint32_t (&wv)[9], const LimbBlock& lb, int (&d)[4]) {
    d[0] = d[1] = d[2] = d[3] = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        const int q = static_cast<int>(wv[1 + w]);
        d[0] = __dp4a(q, static_cast<int>(lb.L[0][w]), d[0]);
        d[1] = __dp4a(q, static_cast<int>(lb.L[1][w]), d[1]);
        d[2] = __dp4a(q, static_cast<int>(lb.L[2][w]), d[2]);
        d[3] = __dp4a(q, static_cast<int>(lb.L[3][w]), d[3]);
    }
}

__device__ __forceinline__ float q8_block_limb(const uint32_t (&wv)[9], const LimbBlock& lb) {
    int d[4];
    q8_block_dsums(wv, lb, d);
    return combine_limbs(d[0], d[1], d[2], d[3]);
}

// Q4: nibbles (0..15, the +8-biased codes) are exact as signed bytes; the bias
// is removed with the plane sums: sum (nib - 8) L = sum nib L - 8 S.
__device__ __forceinline__ void q4_block_dsums(const uint32_t (&qw)[4], const LimbBlock& lb, const int4 S, int (&d)[4]) {
    d[0] = -8 * S.x;
    d[1] = -8 * S.y;
    d[2] = -8 * S.z;
    d[3] = -8 * S.w;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        const int lo = static_cast<int>(qw[w] & 0x0F0F0F0Fu);          // elements 8w + 0, 2, 4, 6
        const int hi = static_cast<int>((qw[w] >> 4) & 0x0F0F0F0Fu);   // elements 8w + 1, 3, 5, 7
        d[0] = __dp4a(lo, static_cast<int>(lb.L[0][2 * w]), d[0]);
        d[1] = __dp4a(lo, static_cast<int>(lb.L[1][2 * w]), d[1]);
        d[2] = __dp4a(lo, static_cast<int>(lb.L[2][2 * w]), d[2]);
        d[3] = __dp4a(lo, static_cast<int>(lb.L[3][2 * w]), d[3]);
        d[0] = __dp4a(hi, static_cast<int>(lb.L[0][2 * w + 1]), d[0]);
        d[1] = __dp4a(hi, static_cast<int>(lb.L[1][2 * w + 1]), d[1]);
        d[2] = __dp4a(hi, static_cast<int>(lb.L[2][2 * w + 1]), d[2]);
        d[3] = __dp4a(hi, static_cast<int>(lb.L[3][2 * w + 1]), d[3]);
    }
}

__device__ __forceinline__ float q4_block_limb(const uint32_t (&qw)[4], const LimbBlock& lb, const int4 S) {
    int d[4];
    q4_block_dsums(qw, lb, S, d);
    return combine_limbs(d[0], d[1], d[2], d[3]);
}

// One thread's share of a block's limbs: elements 8*sub .. 8*sub+7 of the block
// (for Q4 exactly one group of 8 in the 0,2,4,6,1,3,5,7 order).  The four
// threads of a block are lanes 4k..4k+3 of one warp, all active (`act` false
// for padding threads): the group's maximum and plane sums take two shuffles.
// Results: the digit-plane word pairs w[j][0..1] of the 8 elements, the block
// factor cb = 2^(e - 30) (NaN when the block holds a non-finite value) and the
// block's plane sums S_j.
template <uint32_t DT>
__device__ __forceinline__ void limb_part_digits(const float4 a, const float4 b, bool act, uint32_t (&w)[4][2],
                                                 float& cb_out, int (&S)[4]) {
    const float xv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    float amax = 0.0f;
    uint32_t bad = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        amax = fmaxf(amax, fabsf(xv[i]));
        bad |= isfinite(xv[i]) ? 0u : 1u;
    }
    if (!act) {
        amax = 0.0f;
        bad = 0u;
    }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
        bad |= __shfl_xor_sync(0xFFFFFFFFu, bad, o);
    }
    // e with max |x| (1 + 2^-8) < 2^e, from the exponent bits of t = max |x| * (1 + 2^-8):
    // t in [2^(tb-127), 2^(tb-126)), e = tb - 126.  2^(30-e) and 2^(e-30) come from
    // exponent bits where both are normal floats; otherwise (blocks near the ends of
    // the range) each x is scaled by ldexpf.
    const bool live = amax > 0.0f && !bad;
    const float t = amax * 1.00390625f;
    const uint32_t tb = __float_as_uint(t) >> 23;
    int e = 0;
    float up = 0.0f, cb = 0.0f;
    bool slow = false;
    if (live) {
        if (tb >= 30u && tb <= 254u) {
            up = __uint_as_float((283u - tb) << 23);   // 2^(30 - e)
            cb = __uint_as_float((tb - 29u) << 23);    // 2^(e - 30)
        } else {
            if (tb > 254u) e = 128;   // t overflowed: max |x| < 2^128
            else frexpf(t, &e);       // t < 2^e
            slow = true;
            cb = ldexpf(1.0f, e - 30);
        }
    }
    // U = X + 0x80808080 per element, in record order (Q4: 0,2,4,6 then 1,3,5,7)
    uint32_t u[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int src = (DT == kDtypeQ4) ? ((i & 3) * 2 + (i >> 2)) : i;
        const int X = live ? __float2int_rn(slow ? ldexpf(xv[src], 30 - e) : xv[src] * up) : 0;
        u[i] = static_cast<uint32_t>(X) + 0x80808080u;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) S[j] = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {   // 4 x 4 byte transpose: byte k of element word i -> byte i of plane word 3-k
        const uint32_t t0 = __byte_perm(u[4 * h + 0], u[4 * h + 1], 0x5140u), t1 = __byte_perm(u[4 * h + 0], u[4 * h + 1], 0x7362u);
        const uint32_t t2 = __byte_perm(u[4 * h + 2], u[4 * h + 3], 0x5140u), t3 = __byte_perm(u[4 * h + 2], u[4 * h + 3], 0x7362u);
        w[3][h] = __byte_perm(t0, t2, 0x5410u) ^ 0x80808080u;
        w[2][h] = __byte_perm(t0, t2, 0x7632u) ^ 0x80808080u;
        w[1][h] = __byte_perm(t1, t3, 0x5410u) ^ 0x80808080u;
        w[0][h] = __byte_perm(t1, t3, 0x7632u) ^ 0x80808080u;
#pragma unroll
        for (int j = 0; j < 4; ++j) S[j] = __dp4a(static_cast<int>(w[j][h]), 0x01010101, S[j]);
    }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1)
#pragma unroll
        for (int j = 0; j < 4; ++j) S[j] += __shfl_xor_sync(0xFFFFFFFFu, S[j], o);
    cb_out = bad ? __int_as_float(0x7FC00000) : cb;
}

// The same share stored into a limb record (kLimbRec bytes per block).
template <uint32_t DT>
__device__ __forceinline__ void limb_record_part(const float4 a, const float4 b, bool act, uint8_t* rec, uint32_t sub) {
    uint32_t w[4][2];
    int S[4];
    float cb;
    limb_part_digits<DT>(a, b, act, w, cb, S);
    if (act) {
#pragma unroll
        for (int j = 0; j < 4; ++j) *reinterpret_cast<uint2*>(rec + 32u * j + 8u * sub) = make_uint2(w[j][0], w[j][1]);
        if (sub == 0) {
            *reinterpret_cast<float*>(rec + 128) = cb;
            *reinterpret_cast<int4*>(rec + 144) = make_int4(S[0], S[1], S[2], S[3]);
        }
    }
}

// RMSNorm factor 1 / sqrt(mean(x^2) + eps) of one vector (K floats, K % 4 == 0),
// by all threads of the CTA: the sum of squares in fp64 (so it differs from the
// reference's fp32 running sum by at most that sum's own rounding), then the
// reference's fp32 steps fl(fl(ss / K) + eps), 1 / sqrt (src/nn/ops.cpp:108-113).
// red: 33 doubles of shared memory.
__device__ __forceinline__ float rms_factor(const float* __restrict__ x, uint32_t K, float eps, double* red) {
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5, nw = (blockDim.x + 31u) >> 5;
    double ss = 0.0;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    for (uint32_t i = threadIdx.x; i < K / 4u; i += blockDim.x) {
        const float4 v = __ldcg(x4 + i);
        ss += static_cast<double>(v.x) * v.x + static_cast<double>(v.y) * v.y + static_cast<double>(v.z) * v.z +
              static_cast<double>(v.w) * v.w;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (uint32_t w = 0; w < nw; ++w) t += red[w];
        const float m = __fadd_rn(__fdiv_rn(static_cast<float>(t), static_cast<float>(K)), eps);
        red[32] = static_cast<double>(__fdiv_rn(1.0f, __fsqrt_rn(m)));
    }
    __syncthreads();
    const float r = static_cast<float>(red[32]);
    __syncthreads();   // red is free again
    return r;
}

// x * r * w for 8 consecutive elements starting at element e (the reference's
// order: fl(fl(x r) w)).
__device__ __forceinline__ void rms_apply8(float4& a, float4& b, float r, const float* __restrict__ w, uint32_t e) {
    const float4 wa = __ldg(reinterpret_cast<const float4*>(w + e)), wb = __ldg(reinterpret_cast<const float4*>(w + e) + 1);
    a = make_float4(__fmul_rn(__fmul_rn(a.x, r), wa.x), __fmul_rn(__fmul_rn(a.y, r), wa.y),
                    __fmul_rn(__fmul_rn(a.z, r), wa.z), __fmul_rn(__fmul_rn(a.w, r), wa.w));
    b = make_float4(__fmul_rn(__fmul_rn(b.x, r), wb.x), __fmul_rn(__fmul_rn(b.y, r), wb.y),
                    __fmul_rn(__fmul_rn(b.z, r), wb.z), __fmul_rn(__fmul_rn(b.w, r), wb.w));
}

// Turn the fp32 activations (global memory, read through L2) into limb records
// in shared memory, in one pass, four threads per block; every thread has the
// next round's loads in flight while it converts the current one.  With
// norm_w, each vector is RMS-normalised first (red: 33 doubles of shared memory).
template <uint32_t DT>
__device__ __forceinline__ void stage_limb_records(const float* __restrict__ x, uint32_t K, uint8_t* xsb,
                                                   uint32_t xs_stride, uint32_t M, uint32_t nblk, uint32_t tid,
                                                   uint32_t nthreads, const float* __restrict__ norm_w = nullptr,
                                                   float eps = 0.0f, double* red = nullptr) {
    const uint32_t lane = tid & 31u, sub = lane & 3u;
    const uint32_t tasks = nblk * 4u;   // per vector
    for (uint32_t m = 0; m < M; ++m) {
        const float4* xm = reinterpret_cast<const float4*>(x + static_cast<size_t>(m) * K);
        const float r = norm_w ? rms_factor(x + static_cast<size_t>(m) * K, K, eps, red) : 1.0f;
        uint8_t* recs = xsb + static_cast<size_t>(m) * xs_stride;
        uint32_t base = tid - lane;   // warp-uniform
        float4 na = make_float4(0.f, 0.f, 0.f, 0.f), nb = na;
        if (base + lane < tasks) {
            na = __ldcg(xm + 2u * (base + lane));
            nb = __ldcg(xm + 2u * (base + lane) + 1u);
        }
        for (; base < tasks; base += nthreads) {
            const uint32_t task = base + lane;
            float4 a = na, b = nb;
            if (task + nthreads < tasks) {   // next round in flight
                na = __ldcg(xm + 2u * (task + nthreads));
                nb = __ldcg(xm + 2u * (task + nthreads) + 1u);
            }
            if (norm_w && task < tasks) rms_apply8(a, b, r, norm_w, 8u * task);
            limb_record_part<DT>(a, b, task < tasks, recs + kLimbRec * (task >> 2), sub);
        }
    }
}

// The same records built once per call for every CTA of the matvec that follows
// (global memory, [M][nblk] records of kLimbRec bytes): one thread per 8
// elements over the whole grid.
template <uint32_t DT>
__global__ void __launch_bounds__(256) limb_prep_kernel(const float* __restrict__ x, uint32_t K, uint32_t M,
                                                        uint32_t nblk, uint8_t* __restrict__ recs, uint32_t pdl,
                                                        const float* __restrict__ norm_w, float eps) {
    __shared__ double red[33];
    if (pdl) pdl_wait();
    if (pdl) pdl_launch_dependents();
    const uint32_t tid = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t per = nblk * 4u, total = M * per;
    const bool act = tid < total;
    const uint32_t m = act ? tid / per : 0u, task = act ? tid - m * per : 0u;
    float r = 1.0f;
    if (norm_w) {   // the vectors this CTA's tasks belong to (at most two: the first and the last)
        const uint32_t t0 = blockIdx.x * blockDim.x, t1 = min(t0 + blockDim.x, total) - 1u;
        const uint32_t m0 = t0 / per, m1 = t1 / per;
        const float r0 = rms_factor(x + static_cast<size_t>(m0) * K, K, eps, red);
        const float r1 = m1 == m0 ? r0 : rms_factor(x + static_cast<size_t>(m1) * K, K, eps, red);
        r = m == m1 ? r1 : r0;
    }
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
    if (act) {
        const float4* xm = reinterpret_cast<const float4*>(x + static_cast<size_t>(m) * K);
        a = __ldcg(xm + 2u * task);
        b = __ldcg(xm + 2u * task + 1u);
        if (norm_w) rms_apply8(a, b, r, norm_w, 8u * task);
    }
    limb_record_part<DT>(a, b, act, recs + (static_cast<size_t>(m) * nblk + (task >> 2)) * kLimbRec, task & 3u);
}

// Per-block integer partial sums for verification (qraf_cuda_limb_partials):
// the records are staged as the row kernel stages them, then one warp per row,
// lane = block, writes D[row][block][0..3] and (row 0) c[block].
template <uint32_t DT>
__global__ void __launch_bounds__(256) limb_partials_kernel(const uint8_t* __restrict__ w, uint64_t row_bytes,
                                                            uint32_t N, uint32_t K, uint32_t nblk,
                                                            const float* __restrict__ x, int32_t* __restrict__ d_out,
                                                            float* __restrict__ c_out) {
    extern __shared__ __align__(128) uint8_t smem[];
    stage_limb_records<DT>(x, K, smem, nblk * kLimbRec, 1u, nblk, threadIdx.x, blockDim.x);
    __syncthreads();
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t r = blockIdx.x * (blockDim.x >> 5) + warp;
    if (r >= N) return;
    const uint8_t* row = w + static_cast<size_t>(r) * row_bytes;
    for (uint32_t b = lane; b < nblk; b += 32u) {
        const uint8_t* rec = smem + kLimbRec * b;
        LimbBlock lb;
        lds_limbs(rec, lb);
        int d[4];
        if constexpr (DT == kDtypeQ8) {
            uint32_t wv[9];
            const uint32_t* pw = reinterpret_cast<const uint32_t*>(row + 36u * b);
#pragma unroll
            for (int i = 0; i < 9; ++i) wv[i] = __ldg(pw + i);
            q8_block_dsums(wv, lb, d);
        } else {
            uint32_t qw[4], s16;
            load_q4_block(row, b, qw, s16);
            q4_block_dsums(qw, lb, *reinterpret_cast<const int4*>(rec + 144), d);
        }
        *reinterpret_cast<int4*>(d_out + (static_cast<size_t>(r) * nblk + b) * 4u) = make_int4(d[0], d[1], d[2], d[3]);
        if (r == 0) c_out[b] = *reinterpret_cast<const float*>(rec + 128);
    }
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
// GT: rows per stage, fixed at compile time for FAST (1, 2 or 4; a short last
// stage recomputes its last row instead of branching); 0 for EXACT (runtime p.G).
template <uint32_t DT, bool EXACT, int MT, int GT>
__global__ void __launch_bounds__(kRowThreads, 1) qmv_rows_kernel(const RowParams p) {
    static_assert(MT == 1 || MT == 2, "one or two activation vectors per pass");
    static_assert(EXACT ? GT == 0 : (GT == 1 || GT == 2 || GT == 4), "rows per stage");
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t nst = p.nst;
    uint8_t* slots = smem;
    uint8_t* xsb = smem + static_cast<size_t>(nst) * p.slot_stride;                     // staged activations
    float* pbuf = reinterpret_cast<float*>(xsb + static_cast<size_t>(p.M) * p.xs_stride);   // EXACT only
    float* part = pbuf + (EXACT ? static_cast<size_t>(kRowWarps) * p.G * p.pb_row : 0);    // FAST, several pieces
    const uint32_t part_floats = (!EXACT && p.npieces > 1) ? (p.M * p.part_rows * p.npieces + 1u) & ~1u : 0u;
    uint64_t* full = reinterpret_cast<uint64_t*>(part + part_floats);
    volatile uint32_t* slot_stage = reinterpret_cast<volatile uint32_t*>(full + nst + 1);
    double* red = reinterpret_cast<double*>(full + nst + 1 + (nst + 1) / 2);   // 33 doubles (RMSNorm)

    if (blockDim.x != static_cast<uint32_t>(kRowThreads)) {
        if (threadIdx.x == 0) raise_error(kErrBadLaunch);
        return;
    }
    const uint32_t c = blockIdx.x;
    const uint32_t r0 = (c * p.rows_base + min(c, p.rows_extra)) * p.row_unit;
    const uint32_t nrows = (p.rows_base + (c < p.rows_extra ? 1u : 0u)) * p.row_unit;
    const uint32_t nstages = (nrows + p.G - 1) / p.G * p.npieces;
    constexpr uint32_t kBlockBytes = DT == kDtypeQ8 ? 36u : 18u;

    for (uint32_t s = threadIdx.x; s <= nst; s += kRowThreads) {   // full[nst]: the activation records
        mbar_init(&full[s], 1);
        if (s < nst) slot_stage[s] = 0xFFFFFFFFu;
    }
    fence_mbar_init();
    __syncthreads();
    if (p.pdl) pdl_launch_dependents();

    // Issue one stage's rows into its slot (one lane).  Weights are read-only
    // model data, so the first stages go out before the dependency wait.
    const uint64_t pol = policy_evict_first();
    auto issue = [&](uint32_t s, uint32_t slot) {
        const uint32_t g = p.npieces == 1 ? s : s / p.npieces, pc = s - g * p.npieces;
        const uint32_t rows = min(p.G, nrows - g * p.G);
        const uint32_t a = r0 + g * p.G;   // first (virtual) row of the stage
        uint8_t* dst = slots + static_cast<size_t>(slot) * p.slot_stride;
        if (p.npieces == 1) {   // whole rows: one copy (one per weight where the rows span several)
            const uint32_t bytes = rows * static_cast<uint32_t>(p.row_bytes);
            mbar_arrive_expect_tx(&full[slot], bytes);
            if (p.swiglu) {         // a gate row and an up row: two copies
                for (uint32_t i = 0; i < rows; ++i)
                    bulk_g2s(dst + static_cast<size_t>(i) * p.row_bytes, row_src(p, a + i),
                             static_cast<uint32_t>(p.row_bytes), &full[slot], pol);
            } else if (p.nseg <= 1) {
                bulk_g2s(dst, p.w + static_cast<size_t>(a) * p.row_bytes, bytes, &full[slot], pol);
            } else {
                for (uint32_t i = 0; i < p.nseg; ++i) {
                    const uint32_t lo = max(a, p.seg_row0[i]), hi = min(a + rows, p.seg_row0[i + 1]);
                    if (lo < hi)
                        bulk_g2s(dst + static_cast<size_t>(lo - a) * p.row_bytes, row_src(p, lo),
                                 (hi - lo) * static_cast<uint32_t>(p.row_bytes), &full[slot], pol);
                }
            }
        } else {                // one copy per row of this piece
            const uint32_t pb = min(p.piece_blocks, p.nblk - pc * p.piece_blocks) * kBlockBytes;
            mbar_arrive_expect_tx(&full[slot], rows * pb);
            for (uint32_t i = 0; i < rows; ++i)
                bulk_g2s(dst + i * p.piece_bytes, row_src(p, a + i) + static_cast<size_t>(pc) * p.piece_bytes, pb,
                         &full[slot], pol);
        }
        slot_stage[slot] = s;   // the slot's barrier is now in stage s's phase
    };
    if (lane == 0)
        for (uint32_t s = warp; s < min(min(nst, nstages), p.early); s += kRowWarps) issue(s, s);

    // ── stage the activations (after the previous kernel finished) ──
    // L2-coherent loads (__ldcg): under programmatic dependent launch x may have
    // just been written by the previous kernel, so no L1 copy of it may be trusted.
    if (p.pdl) pdl_wait();
    const uint32_t call = p.world ? *reinterpret_cast<volatile const uint32_t*>(p.seq) + 1u : 0u;
    if constexpr (EXACT) {
        const uint32_t n4 = p.K / 4u;
        for (uint32_t m = 0; m < p.M; ++m) {
            const float4* xm = reinterpret_cast<const float4*>(p.x + static_cast<size_t>(m) * p.K);
            uint8_t* xs = xsb + static_cast<size_t>(m) * p.xs_stride;
            for (uint32_t i = threadIdx.x; i < n4; i += kRowWarps * 32u)
                *reinterpret_cast<float4*>(xs + 144u * (i >> 3) + 16u * (i & 7u)) = __ldcg(xm + i);
        }
    } else if (p.xrec) {
        // records already built: one bulk copy (L2 -> shared memory), completion on full[nst]
        if (threadIdx.x == 0) {
            const uint32_t bytes = p.M * p.nblk * kLimbRec;
            mbar_arrive_expect_tx(&full[nst], bytes);
            for (uint32_t off = 0; off < bytes; off += 32768u)
                bulk_g2s(xsb + off, p.xrec + off, min(32768u, bytes - off), &full[nst], policy_evict_first());
        }
        mbar_wait(&full[nst], 0u);
    } else {
        stage_limb_records<DT>(p.x, p.K, xsb, p.xs_stride, p.M, p.nblk, threadIdx.x, kRowWarps * 32u, p.norm_w,
                               p.norm_eps, red);
    }
    __syncthreads();
    if (lane == 0)   // the rest of the first lap (each warp issues its own stages before it waits on them)
        for (uint32_t s = warp; s < min(nst, nstages); s += kRowWarps)
            if (s >= p.early) issue(s, s);

    // this warp's stages s = warp, warp + 16, ...: ring slot s % nst and phase
    // parity (s / nst) & 1, advanced by subtraction (no division in the loop)
    uint32_t slot = warp % nst, phase = (warp / nst) & 1u;
    for (uint32_t s = warp; s < nstages; s += kRowWarps) {
        if (!wait_stage_id(slot_stage + slot, s)) break;      // error raised; every warp still reaches the end
        if (!mbar_wait(&full[slot], phase)) break;
        const uint32_t sg = p.npieces == 1 ? s : s / p.npieces, pc = s - sg * p.npieces;
        const uint32_t rows_s = min(p.G, nrows - sg * p.G);
        const uint32_t row0 = r0 + sg * p.G;
        const uint32_t pblocks = min(p.piece_blocks, p.nblk - pc * p.piece_blocks), pbase = pc * p.piece_blocks;
        const uint8_t* sb = slots + static_cast<size_t>(slot) * p.slot_stride;

        if constexpr (!EXACT) {
            float racc[GT][MT];
            const uint8_t* rowp[GT];
#pragma unroll
            for (int g = 0; g < GT; ++g) {
                rowp[g] = sb + static_cast<size_t>(min(static_cast<uint32_t>(g), rows_s - 1u)) * p.piece_bytes;
#pragma unroll
                for (int v = 0; v < MT; ++v) racc[g][v] = 0.0f;
            }
            for (uint32_t b = lane; b < pblocks; b += 32u) {   // b: block within the piece
                {
                    LimbBlock lb[MT];
                    float cb[MT];
                    int4 S[MT];
#pragma unroll
                    for (int v = 0; v < MT; ++v) {
                        const uint8_t* rec = xsb + static_cast<size_t>(v) * p.xs_stride + kLimbRec * (pbase + b);
                        lds_limbs(rec, lb[v]);
                        cb[v] = *reinterpret_cast<const float*>(rec + 128);
                        if constexpr (DT == kDtypeQ4) S[v] = *reinterpret_cast<const int4*>(rec + 144);
                    }
                    if constexpr (DT == kDtypeQ8) {
                        uint32_t wv[GT][9];
#pragma unroll
                        for (int g = 0; g < GT; ++g) load_q8_block(rowp[g], b, wv[g]);
#pragma unroll
                        for (int g = 0; g < GT; ++g) {
                            const float sc = __uint_as_float(wv[g][0]);
#pragma unroll
                            for (int v = 0; v < MT; ++v)
                                racc[g][v] = fmaf(q8_block_limb(wv[g], lb[v]), sc * cb[v], racc[g][v]);
                        }
                    } else {
                        uint32_t qw[GT][4], s16[GT];
#pragma unroll
                        for (int g = 0; g < GT; ++g) load_q4_block(rowp[g], b, qw[g], s16[g]);
#pragma unroll
                        for (int g = 0; g < GT; ++g) {
                            const float sc = half_bits_to_float(s16[g]);
#pragma unroll
                            for (int v = 0; v < MT; ++v)
                                racc[g][v] = fmaf(q4_block_limb(qw[g], lb[v], S[v]), sc * cb[v], racc[g][v]);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0 && s + nst < nstages) issue(s + nst, slot);   // the slot's bytes are no longer read
            float tsum[GT][MT];
#pragma unroll
            for (int g = 0; g < GT; ++g)
#pragma unroll
                for (int v = 0; v < MT; ++v) tsum[g][v] = warp_sum(racc[g][v]);
            if (lane == 0) {
#pragma unroll
                for (int g = 0; g < GT; ++g) {
#pragma unroll
                    for (int v = 0; v < MT; ++v) {
                        if (g >= static_cast<int>(rows_s)) continue;
                        if (p.npieces > 1)
                            part[(static_cast<size_t>(v) * p.part_rows + (row0 - r0 + g)) * p.npieces + pc] = tsum[g][v];
                        else if (p.swiglu)
                            { if (g & 1) store_swiglu(p, v, (row0 + g) >> 1, tsum[g > 0 ? g - 1 : 0][v], tsum[g][v]); }
                        else
                            store_out(p, call, v, row0 + g, tsum[g][v]);
                    }
                }
            }
        } else {
            float* pb = pbuf + static_cast<size_t>(warp) * p.G * p.pb_row;
            for (uint32_t m = 0; m < p.M; ++m) {
                const float* xm = reinterpret_cast<const float*>(xsb + static_cast<size_t>(m) * p.xs_stride);
                    for (uint32_t ch = 0; ch < (p.nblk + 31u) / 32u; ++ch) {
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
                    store_out(p, call, m, row0 + lane, total);
                }
                __syncwarp();
            }
            if (lane == 0 && s + nst < nstages) issue(s + nst, slot);
        }
        slot += kRowWarps;
        while (slot >= nst) {
            slot -= nst;
            phase ^= 1u;
        }
    }
    if constexpr (!EXACT) {
        if (p.npieces > 1) {   // rows summed piece by piece, in order
            __syncthreads();
            const uint32_t per = p.swiglu ? nrows >> 1 : nrows;   // outputs per vector: rows, or pairs
            const uint32_t total = p.M * per;
            for (uint32_t i = threadIdx.x; i < total; i += kRowThreads) {
                const uint32_t v = i / per, k = i - v * per;
                const uint32_t rl = p.swiglu ? 2u * k : k;
                const float* pr = part + (static_cast<size_t>(v) * p.part_rows + rl) * p.npieces;
                float t = 0.0f;
                for (uint32_t q = 0; q < p.npieces; ++q) t += pr[q];
                if (!p.swiglu) {
                    store_out(p, call, v, r0 + rl, t);
                    continue;
                }
                float u = 0.0f;
                for (uint32_t q = 0; q < p.npieces; ++q) u += pr[p.npieces + q];
                store_swiglu(p, v, (r0 + rl) >> 1, t, u);
            }
        }
    }
    if (p.world) sharded_gather(p, call);
}

}  // namespace qraf_dev
