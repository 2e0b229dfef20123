// capi.cu — the C ABI of libqraf_cuda.so (declared in include/qraf_cuda.h):
// argument checking, kernel selection and launch planning, the host-pointer
// drop-in entry with its device weight cache, and small host utilities; the
// .qraf model store (model_store.cuh) is included at the end.
#include <algorithm>
#include <atomic>
#include <cudaTypedefs.h>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <random>
#include <string>
#include <tuple>
#include <vector>

#include "common.cuh"
#include "matmul_tc.cuh"
#include "matvec_generic.cuh"
#include "matvec_rows.cuh"
#include "matvec_stream.cuh"
#include "matvec_tc1.cuh"
#include "quantize.cuh"

using namespace qraf_dev;

namespace {

thread_local std::string t_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return code;
}

#define QRAF_CUDA_TRY(expr)                                                                        \
    do {                                                                                           \
        cudaError_t e_ = (expr);                                                                   \
        if (e_ != cudaSuccess) return fail(QRAF_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(e_)); \
    } while (0)

bool known_dtype(uint32_t dt) { return dt == QRAF_DTYPE_Q8_0 || dt == QRAF_DTYPE_Q4_0; }

uint64_t block_bytes_of(uint32_t dt, uint32_t bs) {
    if (dt == QRAF_DTYPE_Q8_0) return 4ull + bs;
    if (dt == QRAF_DTYPE_Q4_0) return 2ull + bs / 2u;
    return 0;
}

// ── per-device state ──────────────────────────────────────────────────────
struct DeviceInfo {
    bool ready = false;
    int sm_count = 0;
    int smem_optin = 0;
};

std::mutex g_dev_mutex;
DeviceInfo g_dev[64];

// Kernels this library has launched in the process (qraf_cuda_launch_count):
// every launch site goes through count_launch() or counted().
std::atomic<uint64_t> g_launches{0};
inline void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
inline cudaError_t counted(cudaError_t e) {
    if (e == cudaSuccess) count_launch();
    return e;
}

constexpr int kSmemReserve = 1024;

// Let `kernel` take up to `bytes` of shared memory per CTA, static included
// (the dynamic limit is what the static arrays leave).
template <typename K>
cudaError_t allow_smem(K kernel, int bytes) {
    cudaFuncAttributes a;
    const cudaError_t e = cudaFuncGetAttributes(&a, kernel);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                bytes - static_cast<int>(a.sharedSizeBytes));
}

int ensure_device(int* dev_out, DeviceInfo** info_out) {
    int dev = 0;
    QRAF_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(QRAF_ERR_INVALID, "device index %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_dev_mutex);
    DeviceInfo& d = g_dev[dev];
    if (!d.ready) {
        cudaDeviceProp prop;
        QRAF_CUDA_TRY(cudaGetDeviceProperties(&prop, dev));
        if (prop.major < 10)
            return fail(QRAF_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a", dev,
                        prop.major, prop.minor);
        d.sm_count = prop.multiProcessorCount;
        d.smem_optin = static_cast<int>(prop.sharedMemPerBlockOptin);
        const int lim = d.smem_optin;
        QRAF_CUDA_TRY(allow_smem(qmv_stream_kernel<kDtypeQ8, true, 1>, lim));
        QRAF_CUDA_TRY(allow_smem(qmv_stream_kernel<kDtypeQ8, false, 1>, lim));
        QRAF_CUDA_TRY(allow_smem(qmv_stream_kernel<kDtypeQ8, false, 2>, lim));
        QRAF_CUDA_TRY(allow_smem(qmv_stream_kernel<kDtypeQ8, false, 4>, lim));
        QRAF_CUDA_TRY(allow_smem(qmv_stream_kernel<kDtypeQ4, true, 1>, lim));
        QRAF_CUDA_TRY(allow_smem(qmv_stream_kernel<kDtypeQ4, false, 1>, lim));
        QRAF_CUDA_TRY(allow_smem(qmv_stream_kernel<kDtypeQ4, false, 2>, lim));
        QRAF_CUDA_TRY(allow_smem(qmv_stream_kernel<kDtypeQ4, false, 4>, lim));
        QRAF_CUDA_TRY(allow_smem(qmv_rows_kernel<kDtypeQ8, true, 1, 0>, lim));
        QRAF_CUDA_TRY(allow_smem(qmv_rows_kernel<kDtypeQ4, true, 1, 0>, lim));
        QRAF_CUDA_TRY(allow_smem(qmv_rows_kernel<kDtypeQ8, false, 1, 1>, lim));
        QRAF_CUDA_TRY(allow_smem(qmv_rows_kernel<kDtypeQ8, false, 1, 2>, lim));
        QRAF_CUDA_TRY(allow_smem(qmv_rows_kernel<kDtypeQ8, false, 1, 4>, lim));
        QRAF_CUDA_TRY(allow_smem(qmv_rows_kernel<kDtypeQ8, false, 2, 2>, lim));
        QRAF_CUDA_TRY(allow_smem(qmv_rows_kernel<kDtypeQ4, false, 1, 1>, lim));
        QRAF_CUDA_TRY(allow_smem(qmv_rows_kernel<kDtypeQ4, false, 1, 2>, lim));
        QRAF_CUDA_TRY(allow_smem(qmv_rows_kernel<kDtypeQ4, false, 1, 4>, lim));
        QRAF_CUDA_TRY(allow_smem(qmv_rows_kernel<kDtypeQ4, false, 2, 2>, lim));
        QRAF_CUDA_TRY(allow_smem(qmv_tc1_kernel<kDtypeQ8>, lim));
        QRAF_CUDA_TRY(allow_smem(qmv_tc1_kernel<kDtypeQ4>, lim));
        QRAF_CUDA_TRY(allow_smem(limb_partials_kernel<kDtypeQ8>, lim));
        QRAF_CUDA_TRY(allow_smem(limb_partials_kernel<kDtypeQ4>, lim));
        QRAF_CUDA_TRY(allow_smem(qmm_tc_kernel<kDtypeQ8, 16>, lim));
        QRAF_CUDA_TRY(allow_smem(qmm_tc_kernel<kDtypeQ8, 32>, lim));
        QRAF_CUDA_TRY(allow_smem(qmm_tc_kernel<kDtypeQ8, 64>, lim));
        QRAF_CUDA_TRY(allow_smem(qmm_tc_kernel<kDtypeQ4, 16>, lim));
        QRAF_CUDA_TRY(allow_smem(qmm_tc_kernel<kDtypeQ4, 32>, lim));
        QRAF_CUDA_TRY(allow_smem(qmm_tc_kernel<kDtypeQ4, 64>, lim));
        d.ready = true;
    }
    if (dev_out) *dev_out = dev;
    if (info_out) *info_out = &d;
    return QRAF_OK;
}

// ── streaming-kernel plan ────────────────────────────────────────────────
struct StreamPlan {
    StreamParams p;
    int grid = 0, threads = 0, MT = 1;
    size_t smem = 0;
};

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool plan_stream(const qraf_weight_t& w, const float* x, float* y, uint32_t M, bool exact, int MT,
                 const DeviceInfo& dev, StreamPlan* out) {
    if (w.block_size != 32 || (w.cols % 32) != 0 || (w.row_bytes % 16) != 0) return false;
    if (!aligned16(w.data) || !aligned16(x) || (w.cols % 4) != 0) return false;
    const uint32_t nblk = w.cols / 32;
    const uint32_t nwk = (nblk + 31) / 32;
    const uint32_t cw_max = (MT == 1) ? 16u : (MT == 2 ? 12u : 8u);
    if (nwk > cw_max) return false;
    const uint32_t P = cw_max / nwk;
    const uint32_t CW = nwk * P;
    const uint32_t unit = (MT == 1) ? 2u * P : P;
    const uint64_t rb = w.row_bytes;
    uint32_t R = unit;
    while (R * rb < 16384 && (R + unit) * rb <= 40960) R += unit;
    while (R > 1 && R * rb > 49152) --R;
    const uint32_t G = std::min<uint32_t>(static_cast<uint32_t>(dev.sm_count), w.rows);
    const uint32_t rows_base = w.rows / G, rows_extra = w.rows % G;
    const uint32_t max_rows = rows_base + (rows_extra ? 1u : 0u);
    R = std::min(R, max_rows);
    const uint32_t slot_stride = static_cast<uint32_t>((R * rb + 127) / 128 * 128);
    uint32_t pb_row, pb_bytes;
    if (exact) {
        pb_row = nblk + 4;
        pb_bytes = R * pb_row * 4u;
    } else if (MT == 1) {
        pb_row = nwk;
        pb_bytes = R * nwk * 4u;
    } else {
        pb_row = nwk;
        pb_bytes = R * M * nwk * 4u;
    }
    const uint32_t pb_stride = (pb_bytes + 127) / 128 * 128;
    const uint32_t per_slot = slot_stride + pb_stride + 20u;
    const int budget = dev.smem_optin - kSmemReserve;
    const uint32_t stages_needed = (max_rows + R - 1) / R;
    uint32_t nst = std::min<uint32_t>(8u, stages_needed);
    while (nst > 1 && static_cast<int>(nst * per_slot + 64) > budget) --nst;
    if (static_cast<int>(nst * per_slot + 64) > budget) return false;

    StreamParams& p = out->p;
    p.w = static_cast<const uint8_t*>(w.data);
    p.x = x;
    p.y = y;
    p.row_bytes = rb;
    p.N = w.rows;
    p.K = w.cols;
    p.M = M;
    p.nblk = nblk;
    p.nwk = nwk;
    p.P = P;
    p.CW = CW;
    p.R = R;
    p.nst = nst;
    p.slot_stride = slot_stride;
    p.pb_stride = pb_stride;
    p.pb_row = pb_row;
    p.rows_base = rows_base;
    p.rows_extra = rows_extra;
    out->grid = static_cast<int>(G);
    out->threads = static_cast<int>((CW + 1) * 32);
    out->MT = MT;
    out->smem = static_cast<size_t>(nst) * (slot_stride + pb_stride) + nst * 20u + 64u;
    return true;
}

// ── row-owner kernel plan (M = 1 or 2 FAST; any M EXACT) ─────────────────
struct RowPlan {
    RowParams p;
    int grid = 0;
    size_t smem = 0;
};

constexpr int kPdlSmemBudget = 227 * 1024;   // one CTA per SM: use the whole shared memory

bool rows_eligible(const qraf_weight_t& w, const float* x) {
    return w.block_size == 32 && (w.cols % 32) == 0 && w.cols > 0 && (w.row_bytes % 16) == 0 && aligned16(w.data) &&
           aligned16(x);
}

// Plan one launch over `mcount` activation vectors.  Returns false when the
// staged activations do not fit in shared memory.  pairs: SwiGLU launch (the
// rows are (gate, up) pairs; CTAs take whole pairs, stages hold one pair).
bool plan_rows(const qraf_weight_t& w, const float* x, float* y, uint32_t mcount, bool exact, const DeviceInfo& dev,
               RowPlan* out, bool pairs = false) {
    const uint32_t nblk = w.cols / 32;
    const uint64_t rb = w.row_bytes;
    const uint32_t unit = pairs ? 2u : 1u, units = w.rows / unit;
    const uint32_t grid = std::min<uint32_t>(static_cast<uint32_t>(dev.sm_count), units);
    const uint32_t rows_base = units / grid, rows_extra = units % grid;   // in units of `unit` rows
    const uint32_t max_rows = (rows_base + (rows_extra ? 1u : 0u)) * unit;
    const uint32_t bb = w.dtype == QRAF_DTYPE_Q8_0 ? 36u : 18u;
    uint32_t G = 1, piece = nblk, npieces = 1;
    // Rows per stage: enough stages to keep all warps busy, then as many rows as
    // fit ~18 KB (more rows share each staged activation block).  Whole rows.
    while (G < kRowGMax && (2 * G) * rb <= 18432 && 5 * ((max_rows + 2 * G - 1) / (2 * G)) >= 4 * kRowWarps) G *= 2;
    if (!exact && mcount == 2) G = 2;
    // SwiGLU pairs: two pairs per stage where four rows fit the stage (one vector), so
    // that each staged activation record serves four rows; a row's sum does not
    // depend on the rows beside it
    if (pairs) G = (mcount == 1 && 4 * rb <= 18432 && max_rows >= 8) ? 4u : 2u;
    const bool long_rows = 2 * rb > 18432;   // not even 2 whole rows per stage
    if (!exact && long_rows) {
        // FAST, long rows: stages of 4 rows (2 for two vectors) x one piece of K, so
        // that each staged activation block serves several rows; each stage leaves
        // its partial sums in shared memory and rows are summed piece by piece, in
        // order, at the end.  The pieces depend on K and the dtype only, so a row's
        // arithmetic is the same however the rows are spread over CTAs or GPUs
        // (row shards give the unsharded bits).
        G = (mcount == 2 || pairs) ? 2u : 4u;
        while (!pairs && G > 1 && G > max_rows) G >>= 1;
        const uint32_t cap = 18432u / (4u * bb) / 8u * 8u;   // blocks per piece at 4 rows per ~18 KB stage
        npieces = (nblk + cap - 1) / cap;
        piece = ((nblk + npieces - 1) / npieces + 7u) / 8u * 8u;
        npieces = (nblk + piece - 1) / piece;
    }
    const uint32_t rec = exact ? 144u : kLimbRec;      // bytes per staged 32-element block
    const uint64_t x_bytes = static_cast<uint64_t>(mcount) * nblk * rec;
    const uint32_t pb_row = nblk + 4;
    const uint64_t pb_bytes = exact ? static_cast<uint64_t>(kRowWarps) * G * pb_row * 4u : 0;
    const uint64_t budget = std::min<uint64_t>(kPdlSmemBudget, static_cast<uint64_t>(dev.smem_optin - kSmemReserve));
    uint32_t piece_bytes = 0, slot_stride = 0, nst = 0;
    uint64_t fixed = 0;
    auto layout = [&]() {
        npieces = (nblk + piece - 1) / piece;
        if (npieces == 1) piece = nblk;
        piece_bytes = piece * bb;
        slot_stride = static_cast<uint32_t>(((npieces == 1 ? G * rb : static_cast<uint64_t>(G) * piece_bytes) + 127) / 128 * 128);
        const uint64_t part_bytes = npieces > 1 ? ((static_cast<uint64_t>(mcount) * max_rows * npieces + 1) & ~1ull) * 4u : 0;
        const uint32_t stages = (max_rows + G - 1) / G * npieces;
        fixed = x_bytes + pb_bytes + part_bytes + 64 + 272;   // + the RMSNorm reduction buffer
        nst = budget <= fixed ? 0u
                              : static_cast<uint32_t>(std::min<uint64_t>({32u, stages, (budget - fixed) / (slot_stride + 12u)}));
    };
    layout();
    if (nst == 0) return false;
    RowParams& p = out->p;
    p.w = static_cast<const uint8_t*>(w.data);
    p.x = x;
    p.y = y;
    p.row_bytes = rb;
    p.N = w.rows;
    p.K = w.cols;
    p.M = mcount;
    p.nblk = nblk;
    p.G = G;
    p.piece_blocks = piece;
    p.npieces = npieces;
    p.piece_bytes = piece_bytes;
    p.part_rows = max_rows;
    p.nst = nst;
    p.slot_stride = slot_stride;
    p.xs_stride = nblk * rec;
    p.pb_row = pb_row;
    p.rows_base = rows_base;
    p.rows_extra = rows_extra;
    p.row_unit = unit;
    p.swiglu = 0;
    p.accumulate = 0;
    p.norm_w = nullptr;
    p.norm_eps = 0.0f;
    for (int i = 0; i < kMaxSeg; ++i) p.seg_b[i] = nullptr;
    p.pdl = 0;
    p.xrec = nullptr;
    // Ring stages issued before the dependency wait: a few, not the whole first lap.
    // The activation loads and limb records that follow the wait are slowed by the
    // copies in flight (the issuing lanes are held while theirs are served), so the
    // rest of the lap goes out after the activations are staged.  Measured on B200
    // (pipelined launches, against the whole lap early): Q4 4096 x 4096 5.89 -> 5.54
    // us, Q8 4096 x 4096 6.65 -> 6.02, Q8 11008 x 2048 8.99 -> 7.53, Q8 2048 x 11008
    // 11.43 -> 9.50, Q4 28672 x 8192 37.95 -> 35.53; 2, 8 and 12 stages did worse on
    // most shapes, and stages above ~10 KB want 4.
    p.early = std::min<uint32_t>(nst, slot_stride <= 10240u ? 6u : 4u);
    p.nseg = 0;
    for (int i = 0; i < kMaxSeg; ++i) {
        p.seg_w[i] = nullptr;
        p.seg_y[i] = nullptr;
        p.seg_row0[i] = 0;
    }
    p.seg_row0[kMaxSeg] = 0;
    p.world = 0;
    p.rank = 0;
    p.seq = nullptr;
    p.y_ld = w.rows;
    p.row_off = 0;
    p.y_full = nullptr;
    p.v_off = 0;
    p.local_ll = nullptr;
    p.ll_cap = 0;
    p.cta_counter = nullptr;
    for (int r = 0; r < kMaxWorld; ++r) p.peer_ll[r] = nullptr;
    out->grid = static_cast<int>(grid);
    out->smem = static_cast<size_t>(nst) * slot_stride + fixed + nst * 12u;
    return true;
}

template <typename Kern>
cudaError_t launch_ex(Kern kernel, int grid, int threads, size_t smem, cudaStream_t st, bool pdl, const RowParams& p) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(static_cast<unsigned>(threads));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return counted(cudaLaunchKernelEx(&cfg, kernel, p));
}

template <uint32_t DT>
cudaError_t launch_rows_dt(const RowPlan& pl, const RowParams& p, bool exact, int MT, bool pdl, cudaStream_t st) {
    if (exact) return launch_ex(qmv_rows_kernel<DT, true, 1, 0>, pl.grid, kRowThreads, pl.smem, st, pdl, p);
    if (MT == 2) return launch_ex(qmv_rows_kernel<DT, false, 2, 2>, pl.grid, kRowThreads, pl.smem, st, pdl, p);
    if (p.G == 1) return launch_ex(qmv_rows_kernel<DT, false, 1, 1>, pl.grid, kRowThreads, pl.smem, st, pdl, p);
    if (p.G == 2) return launch_ex(qmv_rows_kernel<DT, false, 1, 2>, pl.grid, kRowThreads, pl.smem, st, pdl, p);
    return launch_ex(qmv_rows_kernel<DT, false, 1, 4>, pl.grid, kRowThreads, pl.smem, st, pdl, p);
}

cudaError_t launch_rows(uint32_t dtype, const RowPlan& pl, bool exact, int MT, bool pdl, cudaStream_t st) {
    RowParams p = pl.p;
    p.pdl = pdl ? 1u : 0u;
    return dtype == QRAF_DTYPE_Q8_0 ? launch_rows_dt<kDtypeQ8>(pl, p, exact, MT, pdl, st)
                                    : launch_rows_dt<kDtypeQ4>(pl, p, exact, MT, pdl, st);
}

// kind 0: the kernels' own scratch (one call at a time); kind 1: a buffer that
// lives across the several launches of one call (the SwiGLU entry's up projection).
int stream_scratch(cudaStream_t st, size_t bytes, uint8_t** out, const char* what, int kind = 0);

// FAST row kernel, with the activation limbs built once by limb_prep_kernel (into
// the stream's scratch) when every CTA would otherwise spend a large share of its
// time building them (long K, few rows per CTA: long-K projections, row shards on
// many GPUs); the row kernel then copies the records and waits for the prep kernel
// through programmatic dependent launch (its weight copies start meanwhile).
// Measured on B200 with the early-stage rule (pipelined launches, prep / no prep):
// Q4 2048 x 28672 18.7 / 21.3 us, Q4 8192 x 28672 53.8 / 56.5, Q8 2048 x 11008
// 9.60 / 9.57 alone but 1.80 / 1.87 ms per decode step (its down projection, where
// the dependency wait is long), Q4 8192 x 8192 13.46 / 12.78.
constexpr uint32_t kPrepMinBlocks = 320;   // K >= 10240
constexpr uint32_t kPrepMaxRows = 96;      // rows per CTA

int launch_rows_fast(uint32_t dtype, RowPlan& pl, int MT, bool overlap, cudaStream_t st) {
    if (pl.p.nblk >= kPrepMinBlocks && pl.p.rows_base + (pl.p.rows_extra ? 1u : 0u) <= kPrepMaxRows) {
        const size_t bytes = static_cast<size_t>(pl.p.M) * pl.p.nblk * kLimbRec;
        uint8_t* recs = nullptr;
        const int rc = stream_scratch(st, bytes, &recs, "the FAST path's activation-limb prep (K >= 10240 with few rows per CTA)");
        if (rc) return rc;
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = overlap ? 1 : 0;
        cfg.gridDim = dim3((pl.p.M * pl.p.nblk * 4u + 255u) / 256u);
        cfg.blockDim = dim3(256);
        cfg.stream = st;
        const cudaError_t e = counted(cudaLaunchKernelEx(&cfg, dtype == QRAF_DTYPE_Q8_0 ? limb_prep_kernel<kDtypeQ8> : limb_prep_kernel<kDtypeQ4>,
                                                 pl.p.x, pl.p.K, pl.p.M, pl.p.nblk, recs, overlap ? 1u : 0u,
                                                 pl.p.norm_w, pl.p.norm_eps));
        if (e != cudaSuccess) return fail(QRAF_ERR_CUDA, "limb prep launch: %s", cudaGetErrorString(e));
        pl.p.xrec = recs;
        overlap = true;   // the row kernel waits for the prep kernel, not for the one before it
    }
    const cudaError_t e = launch_rows(dtype, pl, false, MT, overlap, st);
    if (e != cudaSuccess) return fail(QRAF_ERR_CUDA, "row kernel launch: %s", cudaGetErrorString(e));
    return QRAF_OK;
}

template <uint32_t DT>
cudaError_t launch_stream(const StreamPlan& pl, bool exact, cudaStream_t st) {
    if (exact) {
        (qmv_stream_kernel<DT, true, 1><<<pl.grid, pl.threads, pl.smem, st>>>(pl.p), count_launch());
    } else if (pl.MT == 1) {
        (qmv_stream_kernel<DT, false, 1><<<pl.grid, pl.threads, pl.smem, st>>>(pl.p), count_launch());
    } else if (pl.MT == 2) {
        (qmv_stream_kernel<DT, false, 2><<<pl.grid, pl.threads, pl.smem, st>>>(pl.p), count_launch());
    } else {
        (qmv_stream_kernel<DT, false, 4><<<pl.grid, pl.threads, pl.smem, st>>>(pl.p), count_launch());
    }
    return cudaGetLastError();
}

template <uint32_t DT, bool EXACT, bool PARTIALS>
cudaError_t launch_generic(const GenericParams& gp, uint64_t tasks, cudaStream_t st) {
    const uint64_t grid = (tasks + 7) / 8;
    if (grid == 0) return cudaSuccess;
    if (grid > 0x7FFFFFFFull) return cudaErrorInvalidConfiguration;
    (qmv_generic_kernel<DT, EXACT, PARTIALS><<<static_cast<unsigned>(grid), 256, 0, st>>>(gp), count_launch());
    return cudaGetLastError();
}

// ── tensor-core plan and its scratch memory ──────────────────────────────
// Scratch per call (one launch pair per group of <= 64 vectors): the prepared
// activation tiles, the block factors, the stream-K partial results and the
// tile counters.  The library keeps one scratch area per (device, stream),
// grown on demand; calls on one stream run in order, so they share it safely.
struct TcPlan {
    TcParams p;
    int grid = 0;
    size_t smem = 0;
    uint32_t mv = 0;
    size_t off_part = 0, off_cnt = 0, bytes = 0;   // scratch layout (activation tiles at 0)
};

size_t round256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

bool tc_eligible(const qraf_weight_t& w) {
    return w.block_size == 32 && (w.cols % 32) == 0 && (w.row_bytes % 16) == 0 && aligned16(w.data) && w.rows > 0 &&
           w.cols > 0;
}

// M: vectors of one launch pair (1..64).
constexpr uint64_t kTcMinUnits = 4;

bool plan_tc(const qraf_weight_t& w, uint32_t M, const DeviceInfo& dev, TcPlan* out) {
    if (!tc_eligible(w) || M == 0 || M > kTcMaxVectors) return false;
    const bool q4 = w.dtype == QRAF_DTYPE_Q4_0;
    TcParams& p = out->p;
    p = TcParams{};   // no output fusions unless the caller sets them
    out->mv = M <= 16 ? 16u : (M <= 32 ? 32u : 64u);
    p.w = static_cast<const uint8_t*>(w.data);
    p.row_bytes = w.row_bytes;
    p.N = w.rows;
    p.M = M;
    p.nblk = w.cols / 32u;
    p.n_pad = 2u * out->mv;
    p.act_stride = p.n_pad * 128u + 2u * out->mv * 4u;   // per pair of blocks
    p.unit_blocks = q4 ? 8u : 4u;
    if (p.nblk % p.unit_blocks) return false;
    p.upt = p.nblk / p.unit_blocks;
    p.tiles = (w.rows + kTcRows - 1) / kTcRows;
    const uint64_t units = static_cast<uint64_t>(p.tiles) * p.upt;
    if (units > 0xFFFFFFFFull / static_cast<uint64_t>(dev.sm_count)) return false;
    p.units = static_cast<uint32_t>(units);
    // Rings in stages of two blocks: accumulators (2 x n_pad TMEM columns each),
    // weight codes (16 KB each), activation tiles (n_pad x 128 bytes, from L2, so
    // deep), scales and factors; then as many raw units (18 KB) as fit, up to 8.
    p.nd = std::min(8u, kTcTmemCols / (2u * p.n_pad));
    p.nab = 4;
    p.ns = 16;
    p.nf = 16;
    p.pdl = 1;
    // at least kTcMinUnits units per CTA: fewer CTAs share a tile, so its stream-K
    // combine is shorter (measured on B200: Q8 2048 x 2048 at 8 vectors 17.4 ->
    // 14.1 us, 2560 x 2048 17.0 -> 14.5; large shapes, with many units per SM, unchanged)
    out->grid = static_cast<int>(std::min<uint64_t>(dev.sm_count, std::max<uint64_t>(1u, units / kTcMinUnits)));
    const size_t avail = static_cast<size_t>(dev.smem_optin) - kSmemReserve;
    const uint32_t tile_bytes = p.n_pad * 128u;
    auto layout = [&](uint32_t nraw, uint32_t nbb) {
        return 1024u + static_cast<size_t>(nraw) * kTcRawSlot + p.nab * kTcASlot + static_cast<size_t>(nbb) * tile_bytes +
               p.ns * 2u * kTcRows * 4u + p.nf * 2u * out->mv * 4u +
               8u * (2u * nraw + p.nab + nbb + 32u + p.nd + 2u * p.ns + 2u * p.nf + 2u) + 16u;
    };
    p.nbb = 16;
    p.nraw = 8;
    while (p.nraw > 4 && layout(p.nraw, p.nbb) > avail) --p.nraw;
    while (p.nbb > 4 && layout(p.nraw, p.nbb) > avail) p.nbb -= 2;   // ring depths stay even (pairs of stages)
    while (p.nraw > 2 && layout(p.nraw, p.nbb) > avail) --p.nraw;
    if (layout(p.nraw, p.nbb) > avail) return false;
    out->smem = layout(p.nraw, p.nbb);
    // One CTA per SM: the kernel takes all 512 TMEM columns, so a second CTA on
    // the SM would only wait for them.
    out->smem = std::max<size_t>(out->smem, 120u * 1024u);
    if (out->smem + kSmemReserve > static_cast<size_t>(dev.smem_optin)) return false;
    out->off_part = round256(static_cast<size_t>(p.nblk / 2u) * p.act_stride);
    out->off_cnt = out->off_part + round256(static_cast<size_t>(out->grid) * 2u * M * kTcRows * sizeof(float));
    out->bytes = out->off_cnt + round256(static_cast<size_t>(p.tiles) * sizeof(uint32_t));
    return true;
}

// A stream's scratch area is never freed before qraf_cuda_shutdown: CUDA graphs
// captured from the stream (the host entry's own, or a caller's) hold its
// address.  When a call needs more, a larger area (at least twice the old one,
// so the areas kept add up to less than twice the largest) becomes the stream's
// current one and the old area is kept, still valid for the graphs that use it.
struct TcScratch {
    uint8_t* base = nullptr;
    size_t bytes = 0;
    std::vector<uint8_t*> retired;   // earlier areas of this stream, freed at shutdown
};
std::mutex g_scratch_mutex;
std::map<std::tuple<int, cudaStream_t, int>, TcScratch> g_scratch;   // (device, stream, kind)

// `what` names the path that needs the scratch, for the error message.
int stream_scratch(cudaStream_t st, size_t bytes, uint8_t** out, const char* what, int kind) {
    int dev = 0;
    QRAF_CUDA_TRY(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(g_scratch_mutex);
    TcScratch& s = g_scratch[std::make_tuple(dev, st, kind)];
    if (s.bytes < bytes) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        QRAF_CUDA_TRY(cudaStreamIsCapturing(st, &cs));
        if (cs != cudaStreamCaptureStatusNone)
            return fail(QRAF_ERR_UNSUPPORTED, "%s needs %zu bytes of per-stream scratch (this stream has %zu); make a "
                                              "first call of this shape on the stream before capturing it",
                        what, bytes, s.bytes);
        const size_t want = std::max(bytes, 2 * s.bytes);
        uint8_t* fresh = nullptr;
        if (cudaMalloc(&fresh, want) != cudaSuccess) {
            cudaGetLastError();
            return fail(QRAF_ERR_NOMEM, "%s: per-stream scratch of %zu bytes could not be allocated", what, want);
        }
        if (s.base) s.retired.push_back(s.base);
        s.base = fresh;
        s.bytes = want;
    }
    *out = s.base;
    return QRAF_OK;
}

void tc_scratch_release() {
    std::lock_guard<std::mutex> lk(g_scratch_mutex);
    int cur = 0;
    cudaGetDevice(&cur);
    for (auto& kv : g_scratch) {
        cudaSetDevice(std::get<0>(kv.first));
        cudaDeviceSynchronize();
        if (kv.second.base) cudaFree(kv.second.base);
        for (uint8_t* p : kv.second.retired) cudaFree(p);
    }
    cudaSetDevice(cur);
    g_scratch.clear();
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link to libcuda).
PFN_cuTensorMapEncodeTiled_v12000 g_encode_tiled = nullptr;
std::once_flag g_encode_once;

bool encode_tiled(CUtensorMap* map, CUtensorMapDataType type, const void* base, const cuuint64_t (&dims)[2],
                  cuuint64_t stride, const cuuint32_t (&box)[2], CUtensorMapSwizzle swizzle) {
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode_tiled = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    if (!g_encode_tiled) return false;
    const cuuint64_t strides[1] = {stride};
    const cuuint32_t estr[2] = {1, 1};
    return g_encode_tiled(map, type, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool weight_map(const qraf_weight_t& w, CUtensorMap* map) {
    // the weight as [rows][row_bytes / 4] 32-bit words; a box is 128 rows x 144 bytes
    const cuuint64_t dims[2] = {w.row_bytes / 4u, w.rows};
    const cuuint32_t box[2] = {kTcUnitBytes / 4u, kTcRows};
    return encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, w.data, dims, w.row_bytes, box, CU_TENSOR_MAP_SWIZZLE_NONE);
}

// Input fusions of a tensor-core call (TcInput): the prep kernel forms the
// activations from x (silu(x) * up, or RMSNorm(x) with norm_w) on the way.
struct TcInput {
    const float* up = nullptr;       // [M][K]: the input is silu(x) * up
    const float* norm_w = nullptr;   // [K]: the input is RMSNorm(x) * norm_w
    float eps = 0.0f;
};

template <uint32_t DT, uint32_t MV>
cudaError_t launch_tc_mv(const TcPlan& pl, const CUtensorMap& map, const float* x, uint32_t K, bool pdl_prep,
                         cudaStream_t st, const TcInput* in = nullptr) {
    const TcParams& p = pl.p;
    const uint64_t threads = static_cast<uint64_t>(p.nblk) * MV * 32u;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.gridDim = dim3(static_cast<unsigned>((threads + 255) / 256));
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cfg.numAttrs = pdl_prep ? 1 : 0;
    cudaError_t e;
    if (in && (in->up || in->norm_w)) {
        cfg.gridDim = dim3(p.n_pad / 2u, (p.nblk + kTcPrepBlocks - 1u) / kTcPrepBlocks);   // (vector slot, blocks)
        e = counted(cudaLaunchKernelEx(&cfg, tc_prep_fused_kernel<DT>, x, in->up, in->norm_w, in->eps,
                                       const_cast<uint8_t*>(p.act), p.tile_count, p.tiles, K, p.M, p.nblk, p.n_pad,
                                       pdl_prep ? 1u : 0u));
    } else {
        e = counted(cudaLaunchKernelEx(&cfg, tc_prep_kernel<DT>, x, const_cast<uint8_t*>(p.act), p.tile_count, p.tiles,
                                       K, p.M, p.nblk, p.n_pad, pdl_prep ? 1u : 0u));
    }
    if (e != cudaSuccess) return e;
    cfg.gridDim = dim3(static_cast<unsigned>(pl.grid));
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.numAttrs = 1;   // weights stream while the prep kernel runs; activations wait for it
    return counted(cudaLaunchKernelEx(&cfg, qmm_tc_kernel<DT, MV>, map, p));
}

template <uint32_t DT>
cudaError_t launch_tc_dt(const TcPlan& pl, const CUtensorMap& map, const float* x, uint32_t K, bool pdl_prep,
                         cudaStream_t st, const TcInput* in = nullptr) {
    if (pl.mv == 16) return launch_tc_mv<DT, 16>(pl, map, x, K, pdl_prep, st, in);
    if (pl.mv == 32) return launch_tc_mv<DT, 32>(pl, map, x, K, pdl_prep, st, in);
    return launch_tc_mv<DT, 64>(pl, map, x, K, pdl_prep, st, in);
}

// Fusions of a tensor-core call: the input's (TcInput) and the outputs' (the
// TcParams fields of the same names): weights back to back in memory as
// segments with their own outputs and biases, a bias for a single weight, the
// residual add.
struct TcFusion {
    TcInput in;
    uint32_t nseg = 0;
    float* seg_y[kMaxSeg] = {};
    const float* seg_b[kMaxSeg] = {};
    uint32_t seg_row0[kMaxSeg + 1] = {};
    bool accumulate = false;
};

// Y = W X on the tensor cores, in groups of up to 64 vectors, with scratch at
// `scratch` (pl.bytes for the largest group; nullptr: the stream's own area).
// A row-sharded tensor-core call: this rank's rows [row_off, row_off + rows) of a
// y with y_ld rows, gathered through the comm's receive arrays (TcParams).  Every
// group of up to kTcMaxVectors vectors is one numbered call of the comm.
struct TcShard {
    uint32_t world = 0, rank = 0, y_ld = 0, row_off = 0, v_off = 0;
    float* y_full = nullptr;
    unsigned long long* local_ll = nullptr;
    unsigned long long* peer_ll[kMaxWorld] = {};
    uint64_t ll_cap = 0;
    uint32_t* cta_counter = nullptr;
    uint32_t* seq = nullptr;
};

int matmul_tc(const qraf_weight_t& w, const float* x, float* y, uint32_t M, bool overlap, cudaStream_t st,
              const DeviceInfo& dev, uint8_t* scratch, size_t scratch_cap, const TcFusion* fz = nullptr,
              const TcShard* sh = nullptr) {
    TcPlan pl;
    const uint32_t first = std::min(M, kTcMaxVectors);
    if (!plan_tc(w, first, dev, &pl)) return fail(QRAF_ERR_UNSUPPORTED, "no tensor-core plan for this weight");
    CUtensorMap map;
    if (!weight_map(w, &map)) return fail(QRAF_ERR_CUDA, "could not describe the weight to the TMA unit");
    uint8_t* base = scratch;
    if (!base) {
        const int rc = stream_scratch(st, pl.bytes, &base, "the tensor-core path");
        if (rc) return rc;
    } else if (scratch_cap < pl.bytes) {
        return fail(QRAF_ERR_INVALID, "this call needs %zu bytes of scratch, more than the %zu available", pl.bytes,
                    scratch_cap);
    }
    for (uint32_t m0 = 0; m0 < M; m0 += kTcMaxVectors) {
        const uint32_t cnt = std::min(kTcMaxVectors, M - m0);
        TcPlan one;
        if (!plan_tc(w, cnt, dev, &one)) return fail(QRAF_ERR_UNSUPPORTED, "no tensor-core plan for %u vectors", cnt);
        one.p.act = base;
        one.p.partial = reinterpret_cast<float*>(base + one.off_part);
        one.p.tile_count = reinterpret_cast<uint32_t*>(base + one.off_cnt);
        one.p.y = y ? y + static_cast<size_t>(m0) * w.rows : nullptr;
        const float* xm = x + static_cast<size_t>(m0) * w.cols;
        TcInput in;
        if (fz) {
            TcParams& p = one.p;
            p.nseg = fz->nseg;
            p.accumulate = fz->accumulate ? 1u : 0u;
            for (int i = 0; i < kMaxSeg; ++i) {
                p.seg_b[i] = fz->seg_b[i];
                p.seg_y[i] = (fz->nseg > 1 && fz->seg_y[i])
                                 ? fz->seg_y[i] + static_cast<size_t>(m0) * (fz->seg_row0[i + 1] - fz->seg_row0[i])
                                 : nullptr;
            }
            for (int i = 0; i <= kMaxSeg; ++i) p.seg_row0[i] = fz->seg_row0[i];
            in = fz->in;
            if (in.up) in.up += static_cast<size_t>(m0) * w.cols;
        }
        if (sh) {
            TcParams& p = one.p;
            p.world = sh->world;
            p.rank = sh->rank;
            p.y_ld = sh->y_ld;
            p.row_off = sh->row_off;
            p.v_off = sh->v_off + m0;
            p.y_full = sh->y_full;
            p.local_ll = sh->local_ll;
            p.ll_cap = sh->ll_cap;
            for (int r = 0; r < kMaxWorld; ++r) p.peer_ll[r] = sh->peer_ll[r];
            p.cta_counter = sh->cta_counter;
            p.seq = sh->seq;
        }
        const bool pdl_prep = overlap || m0 > 0;
        const cudaError_t e = w.dtype == QRAF_DTYPE_Q8_0
                                  ? launch_tc_dt<kDtypeQ8>(one, map, xm, w.cols, pdl_prep, st, fz ? &in : nullptr)
                                  : launch_tc_dt<kDtypeQ4>(one, map, xm, w.cols, pdl_prep, st, fz ? &in : nullptr);
        if (e != cudaSuccess) return fail(QRAF_ERR_CUDA, "tensor-core launch: %s", cudaGetErrorString(e));
    }
    return QRAF_OK;
}

int check_weight(const qraf_weight_t* w) {
    if (!w) return fail(QRAF_ERR_INVALID, "weight is NULL");
    if (!known_dtype(w->dtype)) return fail(QRAF_ERR_UNSUPPORTED, "dtype %u is not Q8_0 (10) or Q4_0 (20)", w->dtype);
    if (w->block_size == 0) return fail(QRAF_ERR_INVALID, "block_size is 0");
    if (w->dtype == QRAF_DTYPE_Q4_0 && w->block_size < 2)
        return fail(QRAF_ERR_INVALID, "Q4_0 block_size must be at least 2");
    if (w->row_bytes != qraf_row_bytes(w->dtype, w->block_size, w->cols))
        return fail(QRAF_ERR_INVALID, "row_bytes %llu does not match dtype/block_size/cols",
                    static_cast<unsigned long long>(w->row_bytes));
    if (w->rows && w->cols && !w->data) return fail(QRAF_ERR_INVALID, "weight data is NULL");
    return QRAF_OK;
}

constexpr uint32_t kAutoTcMinVectors = 3;

// ── batch-1 tensor-core kernel (qmv_tc1_kernel) ───────────────────────────
// One vector, block size 32, K a multiple of 1024 up to 4096, 16-byte-aligned
// rows and x, and every 32-row CTA of the (virtual) weight resident in one wave.
struct Tc1Plan {
    Tc1Params p;
    int grid = 0;
    size_t smem = 0;
};

bool tc1_shape_ok(const qraf_weight_t& w) {
    return w.block_size == 32 && w.cols > 0 && (w.cols % 1024u) == 0 && w.cols <= 32u * kT1MaxBlocks &&
           (w.row_bytes % 16) == 0 && aligned16(w.data) && w.rows > 0;
}

// ws[0..count): weights of one dtype and K, as one row range.
bool plan_tc1(const qraf_weight_t* ws, uint32_t count, const float* x, float* const* ys, const DeviceInfo& dev,
              Tc1Plan* out) {
    if (count == 0 || count > static_cast<uint32_t>(kMaxSeg) || !aligned16(x)) return false;
    uint64_t total = 0;
    for (uint32_t i = 0; i < count; ++i) {
        if (!tc1_shape_ok(ws[i]) || ws[i].dtype != ws[0].dtype || ws[i].cols != ws[0].cols) return false;
        total += ws[i].rows;
    }
    const uint64_t grid = (total + kT1Rows - 1) / kT1Rows;
    if (grid == 0 || grid > static_cast<uint64_t>(dev.sm_count)) return false;   // one wave, one CTA per SM
    Tc1Params& p = out->p;
    p = Tc1Params{};
    const uint32_t nblk = ws[0].cols / 32u;
    const uint32_t bb = ws[0].dtype == QRAF_DTYPE_Q8_0 ? 36u : 18u;
    uint32_t npc = (nblk * bb + kT1MaxPieceBytes - 1) / kT1MaxPieceBytes;
    while ((nblk / 32u) % npc) ++npc;   // pieces of a whole number of 32-block groups
    p.nseg = count;
    uint32_t row0 = 0;
    for (uint32_t i = 0; i < count; ++i) {
        p.seg_w[i] = static_cast<const uint8_t*>(ws[i].data);
        p.seg_y[i] = ys ? ys[i] : nullptr;
        p.seg_row0[i] = row0;
        row0 += ws[i].rows;
    }
    for (uint32_t i = count; i <= static_cast<uint32_t>(kMaxSeg); ++i) p.seg_row0[i] = row0;
    p.x = x;
    p.row_bytes = ws[0].row_bytes;
    p.N = static_cast<uint32_t>(total);
    p.nblk = nblk;
    p.npc = npc;
    p.pblk = nblk / npc;
    p.piece_bytes = p.pblk * bb;
    const Tc1Layout L = ws[0].dtype == QRAF_DTYPE_Q8_0 ? tc1_layout<kDtypeQ8>(nblk, p.piece_bytes, kT1Rows * npc)
                                                       : tc1_layout<kDtypeQ4>(nblk, p.piece_bytes, kT1Rows * npc);
    out->smem = L.bytes + 1024u;   // slack for the 1024-byte alignment
    if (out->smem > static_cast<size_t>(dev.smem_optin) || L.slots < kT1Warps) return false;
    out->grid = static_cast<int>(grid);
    return true;
}

int launch_tc1(uint32_t dtype, Tc1Plan& pl, bool overlap, cudaStream_t st) {
    pl.p.pdl = overlap ? 1u : 0u;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(pl.grid));
    cfg.blockDim = dim3(kT1Threads);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = overlap ? 1 : 0;
    const cudaError_t e = dtype == QRAF_DTYPE_Q8_0 ? counted(cudaLaunchKernelEx(&cfg, qmv_tc1_kernel<kDtypeQ8>, pl.p))
                                                   : counted(cudaLaunchKernelEx(&cfg, qmv_tc1_kernel<kDtypeQ4>, pl.p));
    if (e != cudaSuccess) return fail(QRAF_ERR_CUDA, "batch-1 tensor-core kernel launch: %s", cudaGetErrorString(e));
    return QRAF_OK;
}

// y = fl(t + y), element by element (the residual add of an unfused projection).
static __global__ void __launch_bounds__(256) residual_add_kernel(float* __restrict__ y, const float* __restrict__ t,
                                                                  size_t n) {
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        y[i] = __fadd_rn(t[i], y[i]);
}

// y = W x, or with accumulate y = fl(W x + y): in the row kernel's store where
// that kernel runs, else through a per-stream buffer and residual_add_kernel.
int matvec_impl(const qraf_weight_t* w, const float* x, float* y, uint32_t M, int mode_in, cudaStream_t st,
                bool accumulate = false) {
    int rc = check_weight(w);
    if (rc) return rc;
    const bool overlap = (mode_in & QRAF_MODE_FLAG_OVERLAP) != 0;
    int mode = mode_in & 0xFF;
    // AUTO: the row kernel for one or two vectors, the tensor-core tile from three
    // (measured on B200: at M = 3 the tile matches or beats the CUDA-core kernels on
    // every BASELINE shape, at M = 2 it is slower on all of them; for one vector the
    // row kernel also beats the batch-1 tensor-core kernel, 5.7 against 7.1 us on
    // Q4_0 4096 x 4096 in a dependent chain)
    if (mode == QRAF_MODE_AUTO) mode = (M >= kAutoTcMinVectors && tc_eligible(*w)) ? QRAF_MODE_TC : QRAF_MODE_FAST;
    if (mode != QRAF_MODE_EXACT && mode != QRAF_MODE_FAST && mode != QRAF_MODE_TC)
        return fail(QRAF_ERR_INVALID, "unknown mode %d", mode_in);
    if (M == 0 || w->rows == 0) return QRAF_OK;
    if (!y) return fail(QRAF_ERR_INVALID, "y is NULL");
    if (w->cols == 0) {   // an empty dot is 0 (quantize.cpp:189-209 with no blocks); x is not read
        if (accumulate) return fail(QRAF_ERR_UNSUPPORTED, "a residual projection needs at least one column");
        QRAF_CUDA_TRY(cudaMemsetAsync(y, 0, static_cast<size_t>(M) * w->rows * sizeof(float), st));
        return QRAF_OK;
    }
    if (!x) return fail(QRAF_ERR_INVALID, "x is NULL");
    DeviceInfo* dev = nullptr;
    rc = ensure_device(nullptr, &dev);
    if (rc) return rc;
    auto accumulate_via_scratch = [&]() -> int {
        const size_t n = static_cast<size_t>(M) * w->rows;
        uint8_t* buf = nullptr;
        int r = stream_scratch(st, n * sizeof(float), &buf, "a residual projection's output", 3);
        if (r) return r;
        r = matvec_impl(w, x, reinterpret_cast<float*>(buf), M, mode_in, st, false);
        if (r) return r;
        const unsigned grid = static_cast<unsigned>(std::min<size_t>((n + 255) / 256, 8u * dev->sm_count));
        (residual_add_kernel<<<grid, 256, 0, st>>>(y, reinterpret_cast<const float*>(buf), n), count_launch());
        QRAF_CUDA_TRY(cudaGetLastError());
        return QRAF_OK;
    };
    if (accumulate && !((mode == QRAF_MODE_EXACT || (mode == QRAF_MODE_FAST && M <= 2)) && rows_eligible(*w, x)))
        return accumulate_via_scratch();
    if (M == 1 && mode == QRAF_MODE_TC) {   // tensor cores for one vector: the batch-1 kernel where it applies
        Tc1Plan t1;
        if (plan_tc1(w, 1, x, &y, *dev, &t1)) return launch_tc1(w->dtype, t1, overlap, st);
    }
    if (mode == QRAF_MODE_TC) {
        if (!tc_eligible(*w))
            return fail(QRAF_ERR_UNSUPPORTED, "the tensor-core path needs block size 32, K a multiple of %u and "
                                              "16-byte-aligned weights", w->dtype == QRAF_DTYPE_Q4_0 ? 256 : 128);
        return matmul_tc(*w, x, y, M, overlap, st, *dev, nullptr, 0);
    }
    const bool exact = (mode == QRAF_MODE_EXACT);

    // Row-owner streaming kernel: EXACT for any M (vectors in groups that fit in
    // shared memory), FAST for one or two vectors.
    if (rows_eligible(*w, x) && (exact || M <= 2)) {
        uint32_t per = M;
        RowPlan pl;
        while (per > 1 && !plan_rows(*w, x, y, per, exact, *dev, &pl)) per = (per + 1) / 2;
        if (plan_rows(*w, x, y, per, exact, *dev, &pl)) {
            for (uint32_t m0 = 0; m0 < M; m0 += per) {
                const uint32_t cnt = std::min(per, M - m0);
                RowPlan one = pl;
                one.p.x = x + static_cast<size_t>(m0) * w->cols;
                one.p.y = y + static_cast<size_t>(m0) * w->rows;
                one.p.M = cnt;
                one.p.accumulate = accumulate ? 1u : 0u;
                const int MT = exact ? 1 : static_cast<int>(cnt);
                if (!exact) {
                    const int rc2 = launch_rows_fast(w->dtype, one, MT, overlap, st);
                    if (rc2) return rc2;
                    continue;
                }
                const cudaError_t e = launch_rows(w->dtype, one, exact, MT, overlap, st);
                if (e != cudaSuccess) return fail(QRAF_ERR_CUDA, "row kernel launch: %s", cudaGetErrorString(e));
            }
            return QRAF_OK;
        }
    }
    if (accumulate) return accumulate_via_scratch();

    // K-split streaming kernel: FAST for three or more vectors.
    StreamPlan pl;
    if (!exact) {
        int MT = (M == 1) ? 1 : (M == 2 ? 2 : 4);
        bool ok = plan_stream(*w, x, y, M, false, MT, *dev, &pl);
        if (!ok && MT == 4) ok = plan_stream(*w, x, y, M, false, MT = 2, *dev, &pl);
        if (ok) {
            const cudaError_t e = (w->dtype == QRAF_DTYPE_Q8_0) ? launch_stream<kDtypeQ8>(pl, false, st)
                                                                 : launch_stream<kDtypeQ4>(pl, false, st);
            if (e != cudaSuccess) return fail(QRAF_ERR_CUDA, "stream kernel launch: %s", cudaGetErrorString(e));
            return QRAF_OK;
        }
    }

    // Generic kernel: any block size, ragged blocks, any alignment.
    GenericParams gp;
    gp.w = static_cast<const uint8_t*>(w->data);
    gp.x = x;
    gp.y = y;
    gp.row_bytes = w->row_bytes;
    gp.N = w->rows;
    gp.K = w->cols;
    gp.M = M;
    gp.bs = w->block_size;
    gp.nblk = (w->cols + w->block_size - 1) / w->block_size;
    gp.block_bytes = static_cast<uint32_t>(block_bytes_of(w->dtype, w->block_size));
    const uint64_t tasks = static_cast<uint64_t>(w->rows) * M;
    cudaError_t e;
    if (w->dtype == QRAF_DTYPE_Q8_0)
        e = exact ? launch_generic<kDtypeQ8, true, false>(gp, tasks, st) : launch_generic<kDtypeQ8, false, false>(gp, tasks, st);
    else
        e = exact ? launch_generic<kDtypeQ4, true, false>(gp, tasks, st) : launch_generic<kDtypeQ4, false, false>(gp, tasks, st);
    if (e != cudaSuccess) return fail(QRAF_ERR_CUDA, "generic kernel launch: %s", cudaGetErrorString(e));
    return QRAF_OK;
}

// ── host-pointer entry: weight cache + staging ───────────────────────────
struct CacheKey {
    const void* ptr;
    uint64_t bytes;
    uint32_t dtype, bs, rows, cols;
    int device;
    bool operator<(const CacheKey& o) const {
        return std::tie(ptr, bytes, dtype, bs, rows, cols, device) <
               std::tie(o.ptr, o.bytes, o.dtype, o.bs, o.rows, o.cols, o.device);
    }
};

struct HostStaging {
    cudaStream_t stream = nullptr;
    float* x_pinned = nullptr;
    float* y_pinned = nullptr;
    float* x_map = nullptr;   // the pinned buffers as device pointers (null: copies go through cudaMemcpyAsync)
    float* y_map = nullptr;
    float* x_dev = nullptr;
    float* y_dev = nullptr;
    size_t x_cap = 0, y_cap = 0;   // in floats
    // the device status word as the call's last kernel took it (pinned host
    // memory; status_map: as a device pointer, or null when the device cannot
    // map host memory, then status_dev is copied into it)
    uint32_t* status_pinned = nullptr;
    uint32_t* status_map = nullptr;
    uint32_t* status_dev = nullptr;
};

std::mutex g_host_mutex;
std::map<CacheKey, qraf_weight_t> g_cache;

// The cached device copy of the host weight (w_host, dtype, bs, rows, cols) on
// `dev`, uploaded on first use.  Called with g_host_mutex held.
int cache_entry(const void* w_host, uint32_t dtype, uint32_t block_size, uint32_t rows, uint32_t cols, int dev,
                std::map<CacheKey, qraf_weight_t>::iterator* out) {
    const uint64_t need = qraf_row_bytes(dtype, block_size, cols) * rows;
    const CacheKey key{w_host, need, dtype, block_size, rows, cols, dev};
    auto it = g_cache.find(key);
    if (it == g_cache.end()) {
        qraf_weight_t w;
        const int rc = qraf_cuda_weight_upload(w_host, need, dtype, block_size, rows, cols, &w);
        if (rc) return rc;
        it = g_cache.emplace(key, w).first;
    }
    *out = it;
    return QRAF_OK;
}
HostStaging g_staging[64];

// Per cached weight, M and mode: a CUDA graph of the call's device work (x in,
// kernels, y out) on the staging stream, captured after a first eager call.
// Graphs hold the staging buffers and the cached weight, so they are dropped
// when either changes.  A null exec records that capture did not succeed.
struct GraphKey {
    CacheKey w;
    uint32_t M;
    int mode;
    bool operator<(const GraphKey& o) const { return std::tie(w, M, mode) < std::tie(o.w, o.M, o.mode); }
};
std::map<GraphKey, cudaGraphExec_t> g_graphs;

void drop_graphs(int device) {
    for (auto it = g_graphs.begin(); it != g_graphs.end();) {
        if (device < 0 || it->first.w.device == device) {
            if (it->second) cudaGraphExecDestroy(it->second);
            it = g_graphs.erase(it);
        } else {
            ++it;
        }
    }
}

int grow(HostStaging& s, size_t xn, size_t yn, int device) {
    if (!s.stream) QRAF_CUDA_TRY(cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking));
    if (!s.status_pinned) {
        if (cudaMallocHost(&s.status_pinned, sizeof(uint32_t)) != cudaSuccess ||
            cudaMalloc(&s.status_dev, sizeof(uint32_t)) != cudaSuccess)
            return fail(QRAF_ERR_NOMEM, "status word allocation failed");
        if (cudaHostGetDevicePointer(reinterpret_cast<void**>(&s.status_map), s.status_pinned, 0) != cudaSuccess)
            s.status_map = nullptr;
        cudaGetLastError();
    }
    if (xn > s.x_cap || yn > s.y_cap) drop_graphs(device);   // they hold the old buffers
    if (xn > s.x_cap) {
        if (s.x_pinned) cudaFreeHost(s.x_pinned);
        if (s.x_dev) cudaFree(s.x_dev);
        s.x_pinned = nullptr;
        s.x_map = nullptr;
        s.x_dev = nullptr;
        s.x_cap = 0;
        if (cudaMallocHost(&s.x_pinned, xn * sizeof(float)) != cudaSuccess ||
            cudaMalloc(&s.x_dev, xn * sizeof(float)) != cudaSuccess)
            return fail(QRAF_ERR_NOMEM, "staging allocation of %zu floats failed", xn);
        s.x_cap = xn;
        if (cudaHostGetDevicePointer(reinterpret_cast<void**>(&s.x_map), s.x_pinned, 0) != cudaSuccess) s.x_map = nullptr;
        cudaGetLastError();
    }
    if (yn > s.y_cap) {
        if (s.y_pinned) cudaFreeHost(s.y_pinned);
        if (s.y_dev) cudaFree(s.y_dev);
        s.y_pinned = nullptr;
        s.y_map = nullptr;
        s.y_dev = nullptr;
        s.y_cap = 0;
        if (cudaMallocHost(&s.y_pinned, yn * sizeof(float)) != cudaSuccess ||
            cudaMalloc(&s.y_dev, yn * sizeof(float)) != cudaSuccess)
            return fail(QRAF_ERR_NOMEM, "staging allocation of %zu floats failed", yn);
        s.y_cap = yn;
        if (cudaHostGetDevicePointer(reinterpret_cast<void**>(&s.y_map), s.y_pinned, 0) != cudaSuccess) s.y_map = nullptr;
        cudaGetLastError();
    }
    return QRAF_OK;
}

}  // namespace

// ══ exported C ABI ════════════════════════════════════════════════════════
extern "C" {

const char* qraf_cuda_version(void) { return "qraf_b200 0.1 (sm_100a)"; }

int qraf_cuda_init(int device) {
    QRAF_CUDA_TRY(cudaSetDevice(device));
    return ensure_device(nullptr, nullptr);
}

uint64_t qraf_cuda_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int qraf_cuda_last_error(char* buf, size_t len) {
    if (!buf || len == 0) return QRAF_ERR_INVALID;
    const size_t n = std::min(len - 1, t_last_error.size());
    std::memcpy(buf, t_last_error.data(), n);
    buf[n] = '\0';
    return QRAF_OK;
}

int qraf_cuda_device_status(int clear) {
    QRAF_CUDA_TRY(cudaDeviceSynchronize());
    uint32_t v = 0;
    QRAF_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_status, sizeof(v)));
    if (clear) {
        const uint32_t z = 0;
        QRAF_CUDA_TRY(cudaMemcpyToSymbol(g_status, &z, sizeof(z)));
    }
    if (v & kErrWaitTimeout) return fail(QRAF_ERR_TIMEOUT, "a device-side wait expired (status 0x%x)", v);
    if (v & kErrBadLaunch) return fail(QRAF_ERR_INVALID, "a kernel rejected its launch shape (status 0x%x)", v);
    return QRAF_OK;
}

uint64_t qraf_row_bytes(uint32_t dtype, uint32_t block_size, uint32_t cols) {
    if (!known_dtype(dtype) || block_size == 0) return 0;
    const uint64_t nb = (static_cast<uint64_t>(cols) + block_size - 1) / block_size;
    return nb * block_bytes_of(dtype, block_size);
}

static int describe_weight(uint64_t bytes, uint32_t dtype, uint32_t block_size, uint32_t rows, uint32_t cols,
                           qraf_weight_t* out) {
    if (!out) return fail(QRAF_ERR_INVALID, "out is NULL");
    std::memset(out, 0, sizeof(*out));
    if (!known_dtype(dtype)) return fail(QRAF_ERR_UNSUPPORTED, "dtype %u is not Q8_0 (10) or Q4_0 (20)", dtype);
    if (block_size == 0) return fail(QRAF_ERR_INVALID, "block_size is 0");
    if (dtype == QRAF_DTYPE_Q4_0 && block_size < 2) return fail(QRAF_ERR_INVALID, "Q4_0 block_size must be at least 2");
    const uint64_t rb = qraf_row_bytes(dtype, block_size, cols);
    const uint64_t need = rb * rows;
    if (bytes < need)
        return fail(QRAF_ERR_INVALID, "weight holds %llu bytes, %u rows of %llu bytes need %llu",
                    static_cast<unsigned long long>(bytes), rows, static_cast<unsigned long long>(rb),
                    static_cast<unsigned long long>(need));
    int dev = 0;
    QRAF_CUDA_TRY(cudaGetDevice(&dev));
    out->bytes = need;
    out->row_bytes = rb;
    out->dtype = dtype;
    out->block_size = block_size;
    out->rows = rows;
    out->cols = cols;
    out->device = dev;
    return QRAF_OK;
}

int qraf_cuda_weight_wrap(const void* data_dev, uint64_t bytes, uint32_t dtype, uint32_t block_size, uint32_t rows,
                          uint32_t cols, qraf_weight_t* out) {
    int rc = describe_weight(bytes, dtype, block_size, rows, cols, out);
    if (rc) return rc;
    out->data = data_dev;
    return check_weight(out);
}

int qraf_cuda_weight_upload(const void* data_host, uint64_t bytes, uint32_t dtype, uint32_t block_size, uint32_t rows,
                            uint32_t cols, qraf_weight_t* out) {
    int rc = describe_weight(bytes, dtype, block_size, rows, cols, out);
    if (rc) return rc;
    if (!data_host && out->bytes) return fail(QRAF_ERR_INVALID, "host data is NULL");
    void* d = nullptr;
    if (out->bytes) {
        if (cudaMalloc(&d, out->bytes) != cudaSuccess)
            return fail(QRAF_ERR_NOMEM, "cudaMalloc of %llu bytes failed", static_cast<unsigned long long>(out->bytes));
        const cudaError_t e = cudaMemcpy(d, data_host, out->bytes, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            cudaFree(d);
            return fail(QRAF_ERR_CUDA, "weight upload: %s", cudaGetErrorString(e));
        }
    }
    out->data = d;
    out->owned = 1;
    return QRAF_OK;
}

int qraf_cuda_weight_free(qraf_weight_t* w) {
    if (!w) return fail(QRAF_ERR_INVALID, "weight is NULL");
    if (w->owned && w->data) QRAF_CUDA_TRY(cudaFree(const_cast<void*>(w->data)));
    std::memset(w, 0, sizeof(*w));
    return QRAF_OK;
}

int qraf_cuda_weight_shard(const qraf_weight_t* full, uint32_t world, uint32_t rank, qraf_weight_t* out) {
    int rc = check_weight(full);
    if (rc) return rc;
    if (!out || world == 0 || rank >= world) return fail(QRAF_ERR_INVALID, "bad shard %u of %u", rank, world);
    const uint32_t r0 = static_cast<uint32_t>(static_cast<uint64_t>(full->rows) * rank / world);
    const uint32_t r1 = static_cast<uint32_t>(static_cast<uint64_t>(full->rows) * (rank + 1) / world);
    *out = *full;
    out->data = static_cast<const uint8_t*>(full->data) + static_cast<uint64_t>(r0) * full->row_bytes;
    out->rows = r1 - r0;
    out->bytes = static_cast<uint64_t>(out->rows) * full->row_bytes;
    out->owned = 0;
    return QRAF_OK;
}

int qraf_cuda_matvec_q(const qraf_weight_t* w, const float* x_dev, float* y_dev, uint32_t M, int mode, void* stream) {
    return matvec_impl(w, x_dev, y_dev, M, mode, static_cast<cudaStream_t>(stream));
}

static_assert(QRAF_MULTI_MAX_WEIGHTS == kMaxSeg, "the header's weight limit is the kernel's segment count");

// x_out[m] = RMSNorm(x[m]) for the unfused paths (one CTA per vector): with
// `exact` one thread sums the squares in the reference's order, so the result
// is the reference's bits (src/nn/ops.cpp:107-118); otherwise the CTA's fp64 sum.
static __global__ void __launch_bounds__(256) rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w, float eps,
                                                      uint32_t K, float* __restrict__ out, int exact) {
    __shared__ double red[33];
    const float* xm = x + static_cast<size_t>(blockIdx.x) * K;
    float* om = out + static_cast<size_t>(blockIdx.x) * K;
    float r;
    if (exact) {
        if (threadIdx.x == 0) {
            float ss = 0.0f;
            for (uint32_t i = 0; i < K; ++i) ss = __fadd_rn(ss, __fmul_rn(xm[i], xm[i]));
            const float m = __fadd_rn(__fdiv_rn(ss, static_cast<float>(K)), eps);
            red[32] = static_cast<double>(__fdiv_rn(1.0f, __fsqrt_rn(m)));
        }
        __syncthreads();
        r = static_cast<float>(red[32]);
    } else {
        r = rms_factor(xm, K, eps, red);
    }
    for (uint32_t i = threadIdx.x; i < K; i += blockDim.x) om[i] = __fmul_rn(__fmul_rn(xm[i], r), w[i]);
}

// y[m][r] = fl(y[m][r] + b[r]) for the unfused paths.
static __global__ void __launch_bounds__(256) bias_add_kernel(float* __restrict__ y, const float* __restrict__ b, uint32_t rows,
                                                       size_t n) {
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        y[i] = __fadd_rn(y[i], b[i % rows]);
}

// RMSNorm of x into a per-stream buffer (lives across the launches of one call).
static int normalize_into_scratch(const float* x, const float* norm_w, float eps, uint32_t K, uint32_t M, bool exact,
                           cudaStream_t st, const float** out) {
    uint8_t* buf = nullptr;
    const int rc = stream_scratch(st, static_cast<size_t>(M) * K * sizeof(float), &buf,
                                  "the normalised activations of a fused call", 2);
    if (rc) return rc;
    (rmsnorm_kernel<<<M, 256, 0, st>>>(x, norm_w, eps, K, reinterpret_cast<float*>(buf), exact ? 1 : 0), count_launch());
    QRAF_CUDA_TRY(cudaGetLastError());
    *out = reinterpret_cast<const float*>(buf);
    return QRAF_OK;
}

static int add_bias(float* y, const float* b, uint32_t rows, uint32_t M, const DeviceInfo& dev, cudaStream_t st) {
    const size_t n = static_cast<size_t>(M) * rows;
    const unsigned grid = static_cast<unsigned>(std::min<size_t>((n + 255) / 256, 8u * dev.sm_count));
    if (n) (bias_add_kernel<<<grid, 256, 0, st>>>(y, b, rows, n), count_launch());
    QRAF_CUDA_TRY(cudaGetLastError());
    return QRAF_OK;
}

static int multi_impl(const qraf_weight_t* ws, uint32_t count, const float* x_dev, const float* norm_w, float eps,
                      const float* const* biases, float* const* ys_dev, uint32_t M, int mode_in, void* stream) {
    if (!ws || !ys_dev || count == 0 || count > static_cast<uint32_t>(kMaxSeg))
        return fail(QRAF_ERR_INVALID, "multi call needs 1 to %d weights and their outputs", kMaxSeg);
    for (uint32_t i = 0; i < count; ++i) {
        const int rc = check_weight(&ws[i]);
        if (rc) return rc;
        if (ws[i].dtype != ws[0].dtype || ws[i].block_size != ws[0].block_size || ws[i].cols != ws[0].cols ||
            ws[i].device != ws[0].device)
            return fail(QRAF_ERR_INVALID, "weight %u differs from weight 0 in dtype, block size, cols or device", i);
        if (ws[i].rows && !ys_dev[i]) return fail(QRAF_ERR_INVALID, "output %u is NULL", i);
    }
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const bool overlap = (mode_in & QRAF_MODE_FLAG_OVERLAP) != 0;
    int mode = mode_in & 0xFF;
    const bool auto_mode = mode == QRAF_MODE_AUTO;
    if (mode == QRAF_MODE_AUTO) mode = (M >= kAutoTcMinVectors && tc_eligible(ws[0])) ? QRAF_MODE_TC : QRAF_MODE_FAST;
    const bool exact = mode == QRAF_MODE_EXACT;
    bool any_bias = false;
    for (uint32_t i = 0; biases && i < count; ++i) any_bias = any_bias || biases[i] != nullptr;
    const bool fusion = norm_w != nullptr || any_bias;
    if (M == 0) return QRAF_OK;
    if (norm_w && (ws[0].cols % 8u) != 0) return fail(QRAF_ERR_INVALID, "RMSNorm needs K a multiple of 8");
    DeviceInfo* dev = nullptr;
    int rc = ensure_device(nullptr, &dev);
    if (rc) return rc;
    bool tc1_any = false;   // a weight that a call of its own would run on the batch-1 tensor-core kernel
    if (M == 1 && mode == QRAF_MODE_TC && x_dev) {
        Tc1Plan t1;
        if (!fusion && plan_tc1(ws, count, x_dev, ys_dev, *dev, &t1)) return launch_tc1(ws[0].dtype, t1, overlap, st);
        for (uint32_t i = 0; i < count && !tc1_any; ++i)
            tc1_any = ws[i].rows > 0 && plan_tc1(&ws[i], 1, x_dev, &ys_dev[i], *dev, &t1);
    }
    uint64_t total = 0;
    // fused on the row kernel only where each weight alone would run there too, so
    // that the fused launch gives the separate calls' bits
    bool eligible = (exact || (mode == QRAF_MODE_FAST && M <= 2)) && !tc1_any && (count > 1 || fusion) && M > 0 &&
                    ws[0].cols > 0 && x_dev;
    for (uint32_t i = 0; i < count && eligible; ++i) {
        eligible = ws[i].rows > 0 && rows_eligible(ws[i], x_dev);
        total += ws[i].rows;
    }
    if (eligible && total <= 0xFFFFFFFFull) {
        const float* x_in = x_dev;
        const float* fused_norm = norm_w;
        if (norm_w && exact) {   // EXACT normalises first, in the reference's order
            rc = normalize_into_scratch(x_dev, norm_w, eps, ws[0].cols, M, true, st, &x_in);
            if (rc) return rc;
            fused_norm = nullptr;
        }
        qraf_weight_t v = ws[0];   // the weights as one virtual row range
        v.rows = static_cast<uint32_t>(total);
        v.bytes = total * v.row_bytes;
        uint32_t per = M;
        RowPlan pl;
        while (per > 1 && !plan_rows(v, x_in, nullptr, per, exact, *dev, &pl)) per = (per + 1) / 2;
        if (plan_rows(v, x_in, nullptr, per, exact, *dev, &pl)) {
            for (uint32_t m0 = 0; m0 < M; m0 += per) {
                RowPlan one = pl;
                RowParams& p = one.p;
                const uint32_t cnt = std::min(per, M - m0);
                p.x = x_in + static_cast<size_t>(m0) * v.cols;
                p.M = cnt;
                p.norm_w = fused_norm;
                p.norm_eps = eps;
                if (count == 1) {
                    p.nseg = 1;
                    p.w = static_cast<const uint8_t*>(ws[0].data);
                    p.y = ys_dev[0] + static_cast<size_t>(m0) * ws[0].rows;
                    p.seg_b[0] = biases ? biases[0] : nullptr;
                } else {
                    p.nseg = count;
                    uint32_t row0 = 0;
                    for (uint32_t i = 0; i < count; ++i) {
                        p.seg_w[i] = static_cast<const uint8_t*>(ws[i].data);
                        p.seg_y[i] = ys_dev[i] + static_cast<size_t>(m0) * ws[i].rows;
                        p.seg_b[i] = biases ? biases[i] : nullptr;
                        p.seg_row0[i] = row0;
                        row0 += ws[i].rows;
                    }
                    for (uint32_t i = count; i <= static_cast<uint32_t>(kMaxSeg); ++i) p.seg_row0[i] = row0;
                }
                const bool ov = overlap || m0 > 0;
                if (exact) {
                    const cudaError_t e = launch_rows(v.dtype, one, true, 1, ov, st);
                    if (e != cudaSuccess) return fail(QRAF_ERR_CUDA, "row kernel launch: %s", cudaGetErrorString(e));
                } else {
                    rc = launch_rows_fast(v.dtype, one, static_cast<int>(cnt), ov, st);
                    if (rc) return rc;
                }
            }
            return QRAF_OK;
        }
    }
    // otherwise: one call per weight (same results as the fused launch would give),
    // around an RMSNorm pass and bias passes where the call asks for them
    const float* x_in = x_dev;
    if (norm_w) {
        rc = normalize_into_scratch(x_dev, norm_w, eps, ws[0].cols, M, exact, st, &x_in);
        if (rc) return rc;
    }
    const int each = (auto_mode ? QRAF_MODE_AUTO : mode) | (overlap ? QRAF_MODE_FLAG_OVERLAP : 0);
    for (uint32_t i = 0; i < count; ++i) {
        rc = matvec_impl(&ws[i], x_in, ys_dev[i], M, each, st);
        if (rc) return rc;
        if (biases && biases[i]) {
            rc = add_bias(ys_dev[i], biases[i], ws[i].rows, M, *dev, st);
            if (rc) return rc;
        }
    }
    return QRAF_OK;
}

int qraf_cuda_matvec_q_multi(const qraf_weight_t* ws, uint32_t count, const float* x_dev, float* const* ys_dev,
                             uint32_t M, int mode, void* stream) {
    return multi_impl(ws, count, x_dev, nullptr, 0.0f, nullptr, ys_dev, M, mode, stream);
}

int qraf_cuda_matvec_q_multi_ex(const qraf_weight_t* ws, uint32_t count, const float* x_dev, const float* norm_w,
                                float norm_eps, const float* const* biases, float* const* ys_dev, uint32_t M, int mode,
                                void* stream) {
    return multi_impl(ws, count, x_dev, norm_w, norm_eps, biases, ys_dev, M, mode, stream);
}

static int swiglu_impl(const qraf_weight_t* gate, const qraf_weight_t* up, const float* x_dev, const float* norm_w,
                       float eps, float* h_dev, uint32_t M, int mode_in, void* stream) {
    int rc = check_weight(gate);
    if (rc) return rc;
    rc = check_weight(up);
    if (rc) return rc;
    if (gate->dtype != up->dtype || gate->block_size != up->block_size || gate->cols != up->cols ||
        gate->rows != up->rows || gate->device != up->device)
        return fail(QRAF_ERR_INVALID, "gate and up differ in dtype, block size, shape or device");
    if (M == 0 || gate->rows == 0) return QRAF_OK;
    if (!h_dev) return fail(QRAF_ERR_INVALID, "h is NULL");
    if (gate->cols && !x_dev) return fail(QRAF_ERR_INVALID, "x is NULL");
    if (norm_w && (gate->cols % 8u) != 0) return fail(QRAF_ERR_INVALID, "RMSNorm needs K a multiple of 8");
    const int mode = mode_in & 0xFF;
    if (mode != QRAF_MODE_EXACT && mode != QRAF_MODE_FAST && mode != QRAF_MODE_TC && mode != QRAF_MODE_AUTO)
        return fail(QRAF_ERR_INVALID, "unknown mode %d", mode_in);
    const bool overlap = (mode_in & QRAF_MODE_FLAG_OVERLAP) != 0;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    DeviceInfo* dev = nullptr;
    rc = ensure_device(nullptr, &dev);
    if (rc) return rc;
    // fused: FAST (AUTO) for one or two vectors on the row kernel, rows paired
    const bool fast = mode == QRAF_MODE_FAST || (mode == QRAF_MODE_AUTO && M < kAutoTcMinVectors);
    if (fast && M <= 2 && gate->cols > 0 && rows_eligible(*gate, x_dev) && rows_eligible(*up, x_dev) &&
        gate->rows <= 0x7FFFFFFFu) {
        qraf_weight_t v = *gate;   // the pairs as one virtual weight of 2 x rows
        v.rows = 2u * gate->rows;
        v.bytes = static_cast<uint64_t>(v.rows) * v.row_bytes;
        RowPlan pl;
        if (plan_rows(v, x_dev, nullptr, M, false, *dev, &pl, true)) {
            RowParams& p = pl.p;
            p.swiglu = 1;
            p.nseg = 2;
            p.seg_w[0] = static_cast<const uint8_t*>(gate->data);
            p.seg_w[1] = static_cast<const uint8_t*>(up->data);
            p.seg_y[0] = h_dev;
            p.norm_w = norm_w;
            p.norm_eps = eps;
            return launch_rows_fast(v.dtype, pl, static_cast<int>(M), overlap, st);
        }
    }
    // otherwise the reference's steps: [RMSNorm,] gate into h, up into a buffer, h = silu(h) * up
    const float* x_in = x_dev;
    if (norm_w) {
        rc = normalize_into_scratch(x_dev, norm_w, eps, gate->cols, M, mode == QRAF_MODE_EXACT, st, &x_in);
        if (rc) return rc;
    }
    const size_t n = static_cast<size_t>(M) * gate->rows;
    uint8_t* ubuf = nullptr;
    rc = stream_scratch(st, n * sizeof(float), &ubuf, "the SwiGLU entry's up-projection buffer", 1);
    if (rc) return rc;
    rc = matvec_impl(gate, x_in, h_dev, M, mode_in, st);
    if (rc) return rc;
    rc = matvec_impl(up, x_in, reinterpret_cast<float*>(ubuf), M, mode_in, st);
    if (rc) return rc;
    const unsigned grid = static_cast<unsigned>(std::min<size_t>((n + 255) / 256, 8u * dev->sm_count));
    (swiglu_apply_kernel<<<grid, 256, 0, st>>>(h_dev, reinterpret_cast<const float*>(ubuf), n), count_launch());
    QRAF_CUDA_TRY(cudaGetLastError());
    return QRAF_OK;
}

int qraf_cuda_matvec_q_swiglu(const qraf_weight_t* gate, const qraf_weight_t* up, const float* x_dev, float* h_dev,
                              uint32_t M, int mode, void* stream) {
    return swiglu_impl(gate, up, x_dev, nullptr, 0.0f, h_dev, M, mode, stream);
}

int qraf_cuda_matvec_q_swiglu_ex(const qraf_weight_t* gate, const qraf_weight_t* up, const float* x_dev,
                                 const float* norm_w, float norm_eps, float* h_dev, uint32_t M, int mode,
                                 void* stream) {
    return swiglu_impl(gate, up, x_dev, norm_w, norm_eps, h_dev, M, mode, stream);
}

// ── the tensor-core path without allocation ───────────────────────────────
// Its scratch: one fixed array per device, shared by every call on that device.
static __device__ __align__(256) uint8_t g_noalloc_scratch[QRAF_NOALLOC_SCRATCH_BYTES];
static std::mutex g_noalloc_mutex;
static void* g_noalloc_ptr[64] = {};

int qraf_cuda_matmul_tc_noalloc(const qraf_weight_t* w, const float* x_dev, float* y_dev, uint32_t M, int flags,
                                void* stream) {
    int rc = check_weight(w);
    if (rc) return rc;
    if ((flags & ~QRAF_MODE_FLAG_OVERLAP) != 0) return fail(QRAF_ERR_INVALID, "unknown flags 0x%x", flags);
    if (M == 0 || w->rows == 0) return QRAF_OK;
    if (!x_dev || !y_dev) return fail(QRAF_ERR_INVALID, "x or y is NULL");
    if (!tc_eligible(*w))
        return fail(QRAF_ERR_UNSUPPORTED, "the tensor-core path needs block size 32, K a multiple of %u and "
                                          "16-byte-aligned weights", w->dtype == QRAF_DTYPE_Q4_0 ? 256 : 128);
    int dev_index = 0;
    DeviceInfo* dev = nullptr;
    rc = ensure_device(&dev_index, &dev);
    if (rc) return rc;
    TcPlan pl;
    if (!plan_tc(*w, std::min(M, kTcMaxVectors), *dev, &pl))
        return fail(QRAF_ERR_UNSUPPORTED, "no tensor-core plan for this weight");
    if (pl.bytes > QRAF_NOALLOC_SCRATCH_BYTES)
        return fail(QRAF_ERR_INVALID, "this call needs %zu bytes of scratch, more than the %u bytes of the "
                                      "no-allocation scratch array", pl.bytes, QRAF_NOALLOC_SCRATCH_BYTES);
    void* base = nullptr;
    {
        // set-up, once per device, with that device current
        std::lock_guard<std::mutex> lk(g_noalloc_mutex);
        if (!g_noalloc_ptr[dev_index]) {
            const cudaError_t e = cudaGetSymbolAddress(&base, g_noalloc_scratch);
            if (e != cudaSuccess)
                return fail(QRAF_ERR_CUDA, "cudaGetSymbolAddress of the scratch array: %s", cudaGetErrorString(e));
            g_noalloc_ptr[dev_index] = base;
        }
        base = g_noalloc_ptr[dev_index];
    }
    return matmul_tc(*w, x_dev, y_dev, M, (flags & QRAF_MODE_FLAG_OVERLAP) != 0, static_cast<cudaStream_t>(stream),
                     *dev, static_cast<uint8_t*>(base), QRAF_NOALLOC_SCRATCH_BYTES);
}

int qraf_cuda_dot_q(uint32_t dtype, const void* q_dev, const float* x_dev, uint64_t count, uint32_t block_size,
                    float* out_dev, int mode, void* stream) {
    if (count > 0xFFFFFFFFull) return fail(QRAF_ERR_INVALID, "count %llu exceeds 2^32-1", static_cast<unsigned long long>(count));
    qraf_weight_t w;
    const uint64_t rb = qraf_row_bytes(dtype, block_size, static_cast<uint32_t>(count));
    int rc = qraf_cuda_weight_wrap(q_dev, rb, dtype, block_size, 1, static_cast<uint32_t>(count), &w);
    if (rc) return rc;
    return matvec_impl(&w, x_dev, out_dev, 1, mode, static_cast<cudaStream_t>(stream));
}

int qraf_cuda_limb_partials(const qraf_weight_t* w, const float* x_dev, int32_t* d_dev, float* c_dev, void* stream) {
    int rc = check_weight(w);
    if (rc) return rc;
    if (!x_dev || !d_dev || !c_dev) return fail(QRAF_ERR_INVALID, "x, d or c is NULL");
    if (w->block_size != 32 || (w->cols % 32) != 0 || (w->row_bytes % 4) != 0 || (reinterpret_cast<uintptr_t>(w->data) & 3) ||
        (reinterpret_cast<uintptr_t>(x_dev) & 15))
        return fail(QRAF_ERR_UNSUPPORTED, "limb partials need block size 32, K %% 32 == 0, 4-byte rows and a "
                                          "16-byte-aligned x");
    if (w->rows == 0 || w->cols == 0) return QRAF_OK;
    DeviceInfo* dev = nullptr;
    rc = ensure_device(nullptr, &dev);
    if (rc) return rc;
    const uint32_t nblk = w->cols / 32;
    const size_t smem = static_cast<size_t>(nblk) * kLimbRec;
    if (smem + kSmemReserve > static_cast<size_t>(dev->smem_optin))
        return fail(QRAF_ERR_UNSUPPORTED, "K = %u needs %zu bytes of shared memory", w->cols, smem);
    const unsigned grid = (w->rows + 7u) / 8u;
    if (w->dtype == QRAF_DTYPE_Q8_0)
        (limb_partials_kernel<kDtypeQ8><<<grid, 256, smem, static_cast<cudaStream_t>(stream)>>>(
            static_cast<const uint8_t*>(w->data), w->row_bytes, w->rows, w->cols, nblk, x_dev, d_dev, c_dev), count_launch());
    else
        (limb_partials_kernel<kDtypeQ4><<<grid, 256, smem, static_cast<cudaStream_t>(stream)>>>(
            static_cast<const uint8_t*>(w->data), w->row_bytes, w->rows, w->cols, nblk, x_dev, d_dev, c_dev), count_launch());
    QRAF_CUDA_TRY(cudaGetLastError());
    return QRAF_OK;
}

int qraf_cuda_block_partials(const qraf_weight_t* w, const float* x_dev, float* partials_dev, void* stream) {
    int rc = check_weight(w);
    if (rc) return rc;
    if (w->rows == 0 || w->cols == 0) return QRAF_OK;
    if (!x_dev || !partials_dev) return fail(QRAF_ERR_INVALID, "x or partials is NULL");
    rc = ensure_device(nullptr, nullptr);
    if (rc) return rc;
    GenericParams gp;
    gp.w = static_cast<const uint8_t*>(w->data);
    gp.x = x_dev;
    gp.y = partials_dev;
    gp.row_bytes = w->row_bytes;
    gp.N = w->rows;
    gp.K = w->cols;
    gp.M = 1;
    gp.bs = w->block_size;
    gp.nblk = (w->cols + w->block_size - 1) / w->block_size;
    gp.block_bytes = static_cast<uint32_t>(block_bytes_of(w->dtype, w->block_size));
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const cudaError_t e = (w->dtype == QRAF_DTYPE_Q8_0) ? launch_generic<kDtypeQ8, true, true>(gp, w->rows, st)
                                                        : launch_generic<kDtypeQ4, true, true>(gp, w->rows, st);
    if (e != cudaSuccess) return fail(QRAF_ERR_CUDA, "partials kernel launch: %s", cudaGetErrorString(e));
    return QRAF_OK;
}

static int quantize_launch(uint32_t dtype, const float* x, uint64_t rows, uint64_t row_elems, uint32_t bs, void* out,
                           cudaStream_t st) {
    if (!known_dtype(dtype)) return fail(QRAF_ERR_UNSUPPORTED, "dtype %u is not Q8_0 (10) or Q4_0 (20)", dtype);
    if (bs == 0) return fail(QRAF_ERR_INVALID, "block_size is 0");
    if (rows == 0 || row_elems == 0) return QRAF_OK;
    if (!x || !out) return fail(QRAF_ERR_INVALID, "x or out is NULL");
    QuantParams qp;
    qp.x = x;
    qp.out = static_cast<uint8_t*>(out);
    qp.blocks_per_row = (row_elems + bs - 1) / bs;
    qp.nblocks_total = qp.blocks_per_row * rows;
    qp.row_elems = row_elems;
    qp.bs = bs;
    qp.block_bytes = static_cast<uint32_t>(block_bytes_of(dtype, bs));
    const uint64_t grid = (qp.nblocks_total + 255) / 256;
    if (grid > 0x7FFFFFFFull) return fail(QRAF_ERR_INVALID, "too many blocks");
    if (dtype == QRAF_DTYPE_Q8_0)
        (quantize_kernel<kDtypeQ8><<<static_cast<unsigned>(grid), 256, 0, st>>>(qp), count_launch());
    else
        (quantize_kernel<kDtypeQ4><<<static_cast<unsigned>(grid), 256, 0, st>>>(qp), count_launch());
    QRAF_CUDA_TRY(cudaGetLastError());
    return QRAF_OK;
}

int qraf_cuda_quantize(uint32_t dtype, const float* x_dev, uint64_t count, uint32_t block_size, void* out_dev,
                       void* stream) {
    return quantize_launch(dtype, x_dev, 1, count, block_size, out_dev, static_cast<cudaStream_t>(stream));
}

int qraf_cuda_quantize_rows(uint32_t dtype, const float* x_dev, uint32_t rows, uint32_t cols, uint32_t block_size,
                            void* out_dev, void* stream) {
    return quantize_launch(dtype, x_dev, rows, cols, block_size, out_dev, static_cast<cudaStream_t>(stream));
}

int qraf_cuda_dequantize(uint32_t dtype, const void* q_dev, uint64_t count, uint32_t block_size, float* out_dev,
                         void* stream) {
    if (!known_dtype(dtype)) return fail(QRAF_ERR_UNSUPPORTED, "dtype %u is not Q8_0 (10) or Q4_0 (20)", dtype);
    if (block_size == 0) return fail(QRAF_ERR_INVALID, "block_size is 0");
    if (count == 0) return QRAF_OK;
    if (!q_dev || !out_dev) return fail(QRAF_ERR_INVALID, "q or out is NULL");
    const uint64_t nb = (count + block_size - 1) / block_size;
    const uint64_t grid = (nb + 255) / 256;
    const uint32_t bb = static_cast<uint32_t>(block_bytes_of(dtype, block_size));
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (dtype == QRAF_DTYPE_Q8_0)
        (dequantize_kernel<kDtypeQ8><<<static_cast<unsigned>(grid), 256, 0, st>>>(
            static_cast<const uint8_t*>(q_dev), out_dev, count, block_size, bb, nb), count_launch());
    else
        (dequantize_kernel<kDtypeQ4><<<static_cast<unsigned>(grid), 256, 0, st>>>(
            static_cast<const uint8_t*>(q_dev), out_dev, count, block_size, bb, nb), count_launch());
    QRAF_CUDA_TRY(cudaGetLastError());
    return QRAF_OK;
}

// ── row-sharded matvec: comm objects ──────────────────────────────────────
struct qraf_comm {
    int world = 0, rank = 0, device = 0;
    uint64_t cap = 0;
    float* y[QRAF_COMM_BUFFERS] = {};              // this rank's output buffers (used in turn, call by call)
    unsigned long long* ll = nullptr;               // receive array: 2 x cap words, written by the peers
    uint32_t* counter = nullptr;                    // [0]: CTAs finished in the current launch,
                                                    // [32]: calls completed (numbered on the device)
    unsigned long long* peer_ll[QRAF_COMM_MAX_WORLD] = {};
    bool opened = false;
    bool local_group = false;                       // linked by qraf_cuda_comm_open_local (no IPC mappings)
    uint32_t calls = 0;                             // calls issued from the host (picks the output buffer)
};

int qraf_cuda_comm_create(int world, int rank, uint64_t capacity_floats, qraf_comm_t* out) {
    if (!out || world < 1 || world > QRAF_COMM_MAX_WORLD || rank < 0 || rank >= world || capacity_floats == 0)
        return fail(QRAF_ERR_INVALID, "bad comm arguments (world %d, rank %d)", world, rank);
    int rc = ensure_device(nullptr, nullptr);
    if (rc) return rc;
    qraf_comm* c = new qraf_comm();
    c->world = world;
    c->rank = rank;
    cudaGetDevice(&c->device);
    c->cap = capacity_floats;
    bool ok = true;
    for (int b = 0; b < QRAF_COMM_BUFFERS; ++b)
        ok = ok && cudaMalloc(&c->y[b], capacity_floats * sizeof(float)) == cudaSuccess;
    const size_t ll_bytes = 2 * capacity_floats * sizeof(unsigned long long);
    ok = ok && cudaMalloc(&c->ll, ll_bytes) == cudaSuccess && cudaMalloc(&c->counter, 256) == cudaSuccess &&
         cudaMemset(c->ll, 0, ll_bytes) == cudaSuccess && cudaMemset(c->counter, 0, 256) == cudaSuccess &&
         cudaDeviceSynchronize() == cudaSuccess;
    if (!ok) {
        qraf_cuda_comm_destroy(c);
        return fail(QRAF_ERR_NOMEM, "comm buffers of %llu floats could not be allocated",
                    static_cast<unsigned long long>(capacity_floats));
    }
    *out = c;
    return QRAF_OK;
}

int qraf_cuda_comm_handle(qraf_comm_t c, void* handle_out) {
    if (!c || !handle_out) return fail(QRAF_ERR_INVALID, "comm or handle is NULL");
    static_assert(sizeof(cudaIpcMemHandle_t) <= QRAF_COMM_HANDLE_BYTES, "handle size");
    uint8_t* h = static_cast<uint8_t*>(handle_out);
    std::memset(h, 0, QRAF_COMM_HANDLE_BYTES);
    cudaIpcMemHandle_t m;
    QRAF_CUDA_TRY(cudaIpcGetMemHandle(&m, c->ll));
    std::memcpy(h, &m, sizeof(m));
    return QRAF_OK;
}

int qraf_cuda_comm_open(qraf_comm_t c, const void* all_handles) {
    if (!c || !all_handles) return fail(QRAF_ERR_INVALID, "comm or handles is NULL");
    if (c->opened) return fail(QRAF_ERR_INVALID, "comm is already open");
    const uint8_t* h = static_cast<const uint8_t*>(all_handles);
    for (int q = 0; q < c->world; ++q) {
        if (q == c->rank) {
            c->peer_ll[q] = c->ll;
            continue;
        }
        cudaIpcMemHandle_t m;
        std::memcpy(&m, h + static_cast<size_t>(q) * QRAF_COMM_HANDLE_BYTES, sizeof(m));
        void* ptr = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&ptr, m, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) return fail(QRAF_ERR_COMM, "opening rank %d's receive array: %s", q, cudaGetErrorString(e));
        c->peer_ll[q] = static_cast<unsigned long long*>(ptr);
    }
    c->opened = true;
    return QRAF_OK;
}

int qraf_cuda_comm_open_local(qraf_comm_t* comms, int n) {
    if (!comms || n < 1 || n > QRAF_COMM_MAX_WORLD) return fail(QRAF_ERR_INVALID, "bad comm group of %d", n);
    for (int i = 0; i < n; ++i)
        if (!comms[i] || comms[i]->rank != i || comms[i]->world != n || comms[i]->opened)
            return fail(QRAF_ERR_INVALID, "comm %d does not have rank %d of world %d, or is already open", i, i, n);
    int cur = 0;
    cudaGetDevice(&cur);
    for (int i = 0; i < n; ++i) {
        for (int j = 0; j < n; ++j) {
            if (comms[i]->device != comms[j]->device) {
                cudaSetDevice(comms[i]->device);
                const cudaError_t e = cudaDeviceEnablePeerAccess(comms[j]->device, 0);
                if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) {
                    cudaSetDevice(cur);
                    return fail(QRAF_ERR_COMM, "peer access %d -> %d: %s", comms[i]->device, comms[j]->device,
                                cudaGetErrorString(e));
                }
                cudaGetLastError();
            }
            comms[i]->peer_ll[j] = comms[j]->ll;
        }
    }
    cudaSetDevice(cur);
    for (int i = 0; i < n; ++i) {
        comms[i]->opened = true;
        comms[i]->local_group = true;
    }
    return QRAF_OK;
}

int qraf_cuda_comm_destroy(qraf_comm_t c) {
    if (!c) return QRAF_OK;
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(c->device);
    cudaDeviceSynchronize();
    if (c->opened && !c->local_group) {
        for (int q = 0; q < c->world; ++q)
            if (q != c->rank && c->peer_ll[q]) cudaIpcCloseMemHandle(c->peer_ll[q]);
    }
    for (int b = 0; b < QRAF_COMM_BUFFERS; ++b)
        if (c->y[b]) cudaFree(c->y[b]);
    if (c->ll) cudaFree(c->ll);
    if (c->counter) cudaFree(c->counter);
    cudaSetDevice(cur);
    delete c;
    return QRAF_OK;
}

int qraf_cuda_matvec_q_sharded(qraf_comm_t c, const qraf_weight_t* shard, uint32_t total_rows, uint32_t row_offset,
                               const float* x_dev, uint32_t M, int mode_in, void* stream, float** y_out) {
    if (!c || !c->opened) return fail(QRAF_ERR_INVALID, "comm is not open");
    int rc = check_weight(shard);
    if (rc) return rc;
    if (!x_dev || !y_out) return fail(QRAF_ERR_INVALID, "x or y_out is NULL");
    if (M == 0 || shard->rows == 0 || static_cast<uint64_t>(row_offset) + shard->rows > total_rows)
        return fail(QRAF_ERR_INVALID, "rows [%u, %u) outside %u", row_offset, row_offset + shard->rows, total_rows);
    if (static_cast<uint64_t>(M) * total_rows > c->cap)
        return fail(QRAF_ERR_INVALID, "M * total_rows = %llu exceeds the comm capacity %llu",
                    static_cast<unsigned long long>(M) * total_rows, static_cast<unsigned long long>(c->cap));
    const bool overlap = (mode_in & QRAF_MODE_FLAG_OVERLAP) != 0;
    int mode = mode_in & 0xFF;
    // AUTO as for an unsharded call: the tensor-core tile from three vectors
    if (mode == QRAF_MODE_AUTO) mode = (M >= kAutoTcMinVectors && tc_eligible(*shard)) ? QRAF_MODE_TC : QRAF_MODE_FAST;
    if (mode != QRAF_MODE_EXACT && mode != QRAF_MODE_FAST && mode != QRAF_MODE_TC)
        return fail(QRAF_ERR_UNSUPPORTED, "mode %d", mode_in);
    const bool exact = mode == QRAF_MODE_EXACT;
    if (mode == QRAF_MODE_TC) {
        // the tile with the all-gather in its store: one launch pair (one numbered call)
        // per group of up to kTcMaxVectors vectors, each group at its vector offset
        if (!tc_eligible(*shard))
            return fail(QRAF_ERR_UNSUPPORTED, "the tensor-core path needs block size 32, K a multiple of %u and "
                                              "16-byte-aligned weights", shard->dtype == QRAF_DTYPE_Q4_0 ? 256 : 128);
        DeviceInfo* dev = nullptr;
        rc = ensure_device(nullptr, &dev);
        if (rc) return rc;
        const int buf = static_cast<int>(++c->calls % QRAF_COMM_BUFFERS);
        TcShard sh;
        sh.world = static_cast<uint32_t>(c->world);
        sh.rank = static_cast<uint32_t>(c->rank);
        sh.y_ld = total_rows;
        sh.row_off = row_offset;
        sh.y_full = c->y[buf];
        sh.local_ll = c->ll;
        sh.ll_cap = c->cap;
        for (int r = 0; r < c->world; ++r) sh.peer_ll[r] = c->peer_ll[r];
        sh.cta_counter = c->counter;
        sh.seq = c->counter + 32;
        rc = matmul_tc(*shard, x_dev, nullptr, M, overlap, static_cast<cudaStream_t>(stream), *dev, nullptr, 0, nullptr,
                       &sh);
        if (rc) return rc;
        *y_out = c->y[buf];
        return QRAF_OK;
    }
    if (!rows_eligible(*shard, x_dev))
        return fail(QRAF_ERR_UNSUPPORTED, "the sharded path needs block size 32, K a multiple of 32, and 16-byte-aligned "
                                          "rows and pointers");
    DeviceInfo* dev = nullptr;
    rc = ensure_device(nullptr, &dev);
    if (rc) return rc;
    // Vectors in groups of one launch each (FAST: two, the row kernel's widest pass;
    // EXACT: as many as the shared memory takes).  Every launch is one numbered
    // call of the comm's protocol; all of them write into this host call's buffer,
    // each at its own vector offset.
    uint32_t per = exact ? M : std::min<uint32_t>(M, 2u);
    RowPlan pl;
    while (per > 1 && !plan_rows(*shard, x_dev, nullptr, per, exact, *dev, &pl)) per = (per + 1) / 2;
    if (!plan_rows(*shard, x_dev, nullptr, per, exact, *dev, &pl))
        return fail(QRAF_ERR_UNSUPPORTED, "one activation vector of K = %u does not fit one launch", shard->cols);
    const int buf = static_cast<int>(++c->calls % QRAF_COMM_BUFFERS);
    for (uint32_t m0 = 0; m0 < M; m0 += per) {
        RowPlan one = pl;
        RowParams& p = one.p;
        const uint32_t cnt = std::min(per, M - m0);
        p.x = x_dev + static_cast<size_t>(m0) * shard->cols;
        p.M = cnt;
        p.world = static_cast<uint32_t>(c->world);
        p.rank = static_cast<uint32_t>(c->rank);
        p.seq = c->counter + 32;
        p.y_ld = total_rows;
        p.row_off = row_offset;
        p.y_full = c->y[buf];
        p.v_off = m0;
        p.local_ll = c->ll;
        p.ll_cap = c->cap;
        p.cta_counter = c->counter;
        for (int r = 0; r < c->world; ++r) p.peer_ll[r] = c->peer_ll[r];
        // a later group waits for the one before it (it reuses the CTA counter and call number)
        const bool ov = overlap || m0 > 0;
        if (exact) {
            const cudaError_t e = launch_rows(shard->dtype, one, true, 1, ov, static_cast<cudaStream_t>(stream));
            if (e != cudaSuccess) return fail(QRAF_ERR_CUDA, "sharded kernel launch: %s", cudaGetErrorString(e));
        } else {
            rc = launch_rows_fast(shard->dtype, one, static_cast<int>(cnt), ov, static_cast<cudaStream_t>(stream));
            if (rc) return rc;
        }
    }
    *y_out = c->y[buf];
    return QRAF_OK;
}

int qraf_cuda_host_cache_add(const void* w_host, uint64_t w_size, uint32_t dtype, uint32_t block_size,
                             uint32_t out_dim, uint32_t in_dim) {
    if (!known_dtype(dtype)) return fail(QRAF_ERR_UNSUPPORTED, "dtype %u is not Q8_0 (10) or Q4_0 (20)", dtype);
    if (block_size == 0) block_size = 32;   // a null QuantScheme means 32 (backend.cpp:135)
    if (!w_host) return fail(QRAF_ERR_INVALID, "w is NULL");
    if (out_dim == 0) return QRAF_OK;
    const uint64_t need = qraf_row_bytes(dtype, block_size, in_dim) * out_dim;
    if (w_size && w_size < need)
        return fail(QRAF_ERR_INVALID, "weight holds %llu bytes, %u rows need %llu",
                    static_cast<unsigned long long>(w_size), out_dim, static_cast<unsigned long long>(need));
    int dev = 0;
    DeviceInfo* dinfo = nullptr;
    int rc = ensure_device(&dev, &dinfo);
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(g_host_mutex);
    std::map<CacheKey, qraf_weight_t>::iterator it;
    return cache_entry(w_host, dtype, block_size, out_dim, in_dim, dev, &it);
}

int qraf_cuda_host_cache_info(uint32_t* entries, uint64_t* device_bytes) {
    std::lock_guard<std::mutex> lk(g_host_mutex);
    uint64_t b = 0;
    for (const auto& kv : g_cache) b += kv.second.bytes;
    if (entries) *entries = static_cast<uint32_t>(g_cache.size());
    if (device_bytes) *device_bytes = b;
    return QRAF_OK;
}

int qraf_cuda_matvec_q_host(const void* w_host, uint64_t w_size, uint32_t dtype, uint32_t block_size, uint32_t out_dim,
                            uint32_t in_dim, const float* x_host, float* y_host, uint32_t M, int mode) {
    if (M == 0 || out_dim == 0) return QRAF_OK;
    if (!y_host) return fail(QRAF_ERR_INVALID, "y is NULL");
    if (!known_dtype(dtype)) {
        // The reference zero-fills y for a dtype it has no kernel for (backend.cpp:195-198).
        std::memset(y_host, 0, static_cast<size_t>(M) * out_dim * sizeof(float));
        return QRAF_OK;
    }
    if (block_size == 0) block_size = 32;   // a null QuantScheme means 32 (backend.cpp:135)
    if (!w_host || (!x_host && in_dim)) return fail(QRAF_ERR_INVALID, "w or x is NULL");
    int dev = 0;
    DeviceInfo* dinfo = nullptr;
    int rc = ensure_device(&dev, &dinfo);
    if (rc) return rc;
    (void)w_size;   // the reference never reads it either; it reads exactly rows * row_bytes
    std::lock_guard<std::mutex> lk(g_host_mutex);
    std::map<CacheKey, qraf_weight_t>::iterator it;
    rc = cache_entry(w_host, dtype, block_size, out_dim, in_dim, dev, &it);
    if (rc) return rc;
    const CacheKey key = it->first;
    HostStaging& s = g_staging[dev];
    const size_t xn = std::max<size_t>(static_cast<size_t>(M) * in_dim, 4);
    const size_t yn = static_cast<size_t>(M) * out_dim;
    rc = grow(s, xn, yn, dev);
    if (rc) return rc;
    const size_t x_bytes = static_cast<size_t>(M) * in_dim * sizeof(float);
    // the device work of one call: x in, the kernels, y out (all on the staging stream).
    // x and y cross by SM copies of the mapped pinned buffers where the device maps
    // them; the matvec then overlaps its weight prefetch with the copy of x (the
    // copy kernel writes no weight).
    auto sm_copy = [&](bool from_host, const float* src, float* dst, size_t n) -> int {
        const size_t n4 = std::max<size_t>(n / 4, 1);
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = from_host ? 0 : 1;   // y's copy launches under the matvec and waits for it in the kernel
        cfg.gridDim = dim3(static_cast<unsigned>(std::min<size_t>((n4 + 255) / 256, 4u * dinfo->sm_count)));
        cfg.blockDim = dim3(256);
        cfg.stream = s.stream;
        uint32_t* status = from_host ? nullptr : s.status_map;
        QRAF_CUDA_TRY(from_host ? counted(cudaLaunchKernelEx(&cfg, host_copy_kernel<true>, src, dst, n, status))
                                : counted(cudaLaunchKernelEx(&cfg, host_copy_kernel<false>, src, dst, n, status)));
        return QRAF_OK;
    };
    auto enqueue = [&]() -> int {
        int r = QRAF_OK;
        if (in_dim && s.x_map) r = sm_copy(true, s.x_map, s.x_dev, static_cast<size_t>(M) * in_dim);
        else if (in_dim) QRAF_CUDA_TRY(cudaMemcpyAsync(s.x_dev, s.x_pinned, x_bytes, cudaMemcpyHostToDevice, s.stream));
        if (r) return r;
        const int mv_mode = (in_dim && s.x_map) ? (mode | QRAF_MODE_FLAG_OVERLAP) : mode;
        r = matvec_impl(&it->second, s.x_dev, s.y_dev, M, mv_mode, s.stream);
        if (r) return r;
        if (s.y_map && s.status_map) return sm_copy(false, s.y_dev, s.y_map, yn);
        // no mapped host memory: the status word through a one-thread copy kernel, then copy engines
        QRAF_CUDA_TRY(counted(cudaLaunchKernelEx(&(const cudaLaunchConfig_t&)cudaLaunchConfig_t{dim3(1), dim3(1), 0, s.stream,
                                                                                        nullptr, 0},
                                         host_copy_kernel<false>, s.y_dev, s.y_dev, size_t{0}, s.status_dev)));
        QRAF_CUDA_TRY(cudaMemcpyAsync(s.status_pinned, s.status_dev, sizeof(uint32_t), cudaMemcpyDeviceToHost,
                                      s.stream));
        QRAF_CUDA_TRY(cudaMemcpyAsync(s.y_pinned, s.y_dev, yn * sizeof(float), cudaMemcpyDeviceToHost, s.stream));
        return QRAF_OK;
    };
    if (in_dim) std::memcpy(s.x_pinned, x_host, x_bytes);
    *reinterpret_cast<volatile uint32_t*>(s.status_pinned) = 0u;
    const GraphKey gk{key, M, mode};
    auto g = g_graphs.find(gk);
    if (g != g_graphs.end() && g->second) {
        QRAF_CUDA_TRY(cudaGraphLaunch(g->second, s.stream));
    } else {
        rc = enqueue();   // first call: eager (sets up plans and any scratch)
        if (rc) return rc;
    }
    QRAF_CUDA_TRY(cudaStreamSynchronize(s.stream));
    std::memcpy(y_host, s.y_pinned, yn * sizeof(float));
    // the device status word as the copy of y took it: an expired bounded wait in
    // the call's kernels means y is not complete
    const uint32_t status = *reinterpret_cast<volatile uint32_t*>(s.status_pinned);
    if (status & kErrWaitTimeout)
        return fail(QRAF_ERR_TIMEOUT, "a device-side wait expired during this call (status 0x%x); y is incomplete",
                    status);
    if (status & kErrBadLaunch)
        return fail(QRAF_ERR_INVALID, "a kernel rejected its launch shape during this call (status 0x%x)", status);
    if (g == g_graphs.end()) {
        // capture the same work for the next calls with this weight, M and mode
        cudaGraph_t graph = nullptr;
        cudaGraphExec_t exec = nullptr;
        if (cudaStreamBeginCapture(s.stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
            const int crc = enqueue();
            const cudaError_t e = cudaStreamEndCapture(s.stream, &graph);
            if (crc == QRAF_OK && e == cudaSuccess && graph &&
                cudaGraphInstantiate(&exec, graph, 0) != cudaSuccess)
                exec = nullptr;
            if (graph) cudaGraphDestroy(graph);
        }
        cudaGetLastError();   // a capture that did not work only means eager calls
        g_graphs.emplace(gk, exec);
    }
    return QRAF_OK;
}

int qraf_cuda_host_cache_clear(void) {
    std::lock_guard<std::mutex> lk(g_host_mutex);
    drop_graphs(-1);
    int cur = 0;
    cudaGetDevice(&cur);
    for (auto& kv : g_cache) {
        cudaSetDevice(kv.first.device);
        qraf_cuda_weight_free(&kv.second);
    }
    g_cache.clear();
    cudaSetDevice(cur);
    return QRAF_OK;
}

int qraf_cuda_shutdown(void) {
    qraf_cuda_host_cache_clear();
    tc_scratch_release();
    std::lock_guard<std::mutex> lk(g_host_mutex);
    int cur = 0;
    cudaGetDevice(&cur);
    for (int d = 0; d < 64; ++d) {
        HostStaging& s = g_staging[d];
        if (!s.stream && !s.x_dev && !s.y_dev) continue;
        cudaSetDevice(d);
        if (s.x_pinned) cudaFreeHost(s.x_pinned);
        if (s.y_pinned) cudaFreeHost(s.y_pinned);
        if (s.x_dev) cudaFree(s.x_dev);
        if (s.y_dev) cudaFree(s.y_dev);
        if (s.status_pinned) cudaFreeHost(s.status_pinned);
        if (s.status_dev) cudaFree(s.status_dev);
        if (s.stream) cudaStreamDestroy(s.stream);
        s = HostStaging();
    }
    cudaSetDevice(cur);
    return QRAF_OK;
}

void qraf_fill_normal(uint32_t seed, float mean, float stddev, float* out_host, uint64_t n) {
    std::mt19937 rng(seed);
    std::normal_distribution<float> dist(mean, stddev);
    for (uint64_t i = 0; i < n; ++i) out_host[i] = dist(rng);
}

}  // extern "C"

#include "model_store.cuh"
#include "decoder.cuh"
