// The split plan for callers that cannot allocate device memory.
//
// nb200_fold_split needs scratch from its caller: 16 bytes per (row, chunk) for the chunk states
// the merge reads back. Some callers have no way to provide it -- a host runtime that only hands a
// plugin its input and output buffers, an engine running under a fixed device-memory budget where
// any cudaMalloc would fail or fragment the pool, or code on a path where an allocation call would
// synchronise the device. nb200_fold_split_noalloc serves them: it takes its scratch from a
// fixed-size array compiled into this library, so a call allocates nothing.
//
// What a caller must know:
//  * Capacity: rows * ceil(ncols / chunk_cols) <= NB200_NOALLOC_MAX_STATES (262144 states, 4 MiB).
//    Larger requests are rejected with NB200_ERR_CAPACITY before anything is launched.
//  * Every GPU that loads this library holds the 4 MiB array until the process exits.
//  * The first call on a device looks up the array's device address (cudaGetSymbolAddress, with
//    that device current); make that first call before any stream capture.
//  * All calls share the one array and it keeps the last call's contents. Nothing in it needs to
//    start at zero: every state the merge reads is written by the same call's partial kernel first.
//    Calls whose work overlaps on the GPU (other streams, other host threads) race on the array;
//    serialise them (one stream, or events).
#include <mutex>

#include "fold.cuh"
#include "launch.h"

namespace nb200 {

constexpr int64_t kNoAllocMaxStates = 262144;
static_assert(kNoAllocMaxStates * sizeof(nb200_state) == 4 * 1024 * 1024, "4 MiB of chunk states");

// The scratch array. Host code must not pass this name to a kernel: on the host it is only a
// stand-in symbol, not a device address. noalloc_states() returns the device address.
static __device__ __align__(256) nb200_state g_noalloc_states[kNoAllocMaxStates];

namespace {
std::mutex g_noalloc_mutex;
nb200_state* g_noalloc_ptr[64] = {nullptr};

// Device address of g_noalloc_states on the current device, looked up once per device.
int noalloc_states(nb200_state** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        set_error("nb200_fold_split_noalloc: no usable current CUDA device");
        return NB200_ERR_LAUNCH;
    }
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_ptr[dev] == nullptr) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_states);
        if (e != cudaSuccess || p == nullptr) {
            cudaGetLastError();
            set_error("nb200_fold_split_noalloc: cannot resolve the scratch array on device %d: %s", dev,
                      cudaGetErrorString(e));
            return NB200_ERR_LAUNCH;
        }
        g_noalloc_ptr[dev] = static_cast<nb200_state*>(p);
    }
    *out = g_noalloc_ptr[dev];
    return NB200_OK;
}
}  // namespace

}  // namespace nb200

extern "C" int nb200_fold_split_noalloc(int skeleton, const nb200_params* params, const void* x, int dtype,
                                        int64_t rows, int64_t ncols, int64_t stride_row, int64_t stride_col,
                                        int64_t chunk_cols, void* out, void* stream) {
    using namespace nb200;
    // Requests nb200_fold_split would refuse anyway (bad width, chunk or split capacity) go to it for
    // its own error; only the scratch bound is checked here.
    if (rows > 0 && ncols > 0 && chunk_cols > 0) {
        const int64_t nparts = (ncols + chunk_cols - 1) / chunk_cols;
        if (nparts <= 4096 && rows > kNoAllocMaxStates / nparts) {
            set_error("nb200_fold_split_noalloc: %lld rows x %lld chunks exceed the built-in scratch of %lld "
                      "chunk states; use nb200_fold_split with caller-allocated scratch",
                      (long long)rows, (long long)nparts, (long long)kNoAllocMaxStates);
            return NB200_ERR_CAPACITY;
        }
    }
    nb200_state* states = nullptr;
    if (rows > 0) {
        const int rc = noalloc_states(&states);
        if (rc) return rc;
    }
    return nb200_fold_split(skeleton, params, x, dtype, rows, ncols, stride_row, stride_col, chunk_cols, states,
                            kNoAllocMaxStates * (int64_t)sizeof(nb200_state), out, nullptr, stream);
}
