// dispatch_matvec_q_cuda.cpp — the body of qraf::dispatch_matvec_q on the B200 library.
//
// A QRAF build links this file in place of the scalar body of dispatch_matvec_q
// (src/nn/backend.cpp:131-199): it is compiled with the reference's own headers
// (include/nn/backend.h:31-34 declares the function), backend.cpp is compiled
// with -Ddispatch_matvec_q=dispatch_matvec_q_cpu so that its scalar version keeps
// a different name, and the program links libqraf_cuda.so.  Every caller of the
// seam (do_matvec in src/nn/attention.cpp:56-65 for Q/K/V/O/gate/up/down, the
// quantized LM head in src/nn/transformer.cpp:608-616) then runs on the GPU
// without a source change.
//
// Semantics kept from the scalar body: a null QuantScheme means block size 32
// (backend.cpp:135); an unknown dtype leaves y zeroed (backend.cpp:195-198);
// y is complete when the call returns.  The first call with a given weight
// pointer copies the weight to the GPU and caches it (the reference's weights are
// immutable mmap'd model data, src/qraf/loader.cpp:80).  A CUDA failure is
// logged and thrown as QrafError (include/core/error.h:8-11).
//
// Environment: QRAF_CUDA_MODE=exact (default; bit-identical to the scalar body)
// or fast (int8-limb arithmetic, within the reference's own rounding error).
#include "core/error.h"
#include "core/logging.h"
#include "nn/backend.h"
#include "qraf/format.h"
#include "qraf_cuda.h"

#include <cstdlib>
#include <cstring>
#include <string>

namespace qraf {
namespace {

int cuda_mode() {
    static const int mode = [] {
        const char* m = std::getenv("QRAF_CUDA_MODE");
        const int base = (m && std::strcmp(m, "fast") == 0) ? QRAF_MODE_FAST : QRAF_MODE_EXACT;
        return base | QRAF_MODE_FLAG_OVERLAP;   // weights are never written by the kernels before a matvec
    }();
    return mode;
}

}  // namespace

void dispatch_matvec_q(const void* w_data, u64 w_size, DType w_dtype, const QuantScheme* quant, u32 out_dim,
                       u32 in_dim, const f32* x, f32* y) {
    const uint32_t bs = quant ? quant->block_size : 32u;
    const int rc = qraf_cuda_matvec_q_host(w_data, w_size, static_cast<uint32_t>(w_dtype), bs, out_dim, in_dim, x, y,
                                           1, cuda_mode());
    if (rc != QRAF_OK) {
        char msg[512];
        qraf_cuda_last_error(msg, sizeof msg);
        log::error("dispatch_matvec_q on CUDA failed (%d): %s", rc, msg);
        throw QrafError(std::string("dispatch_matvec_q on CUDA failed: ") + msg);
    }
}

}  // namespace qraf
