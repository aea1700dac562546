// RMSNorm over rows that live in host memory: the rows stream through the device in chunks (of
// ramped sizes at both ends, see ramp_rows), with
// the copy of the next chunk to the device and the copy of the previous chunk back to the host
// running on two helper streams while the current chunk's kernel runs on the caller's stream.
// PCIe moves data both ways at once, so a step costs about one direction's transfer time instead
// of the sum of both. The kernel and the results are those of nb200_rms_norm on the same rows.
//
// Device buffers (caller-owned `work`): gamma, then two input and two output chunk buffers used
// alternately. Ordering per chunk k in buffer slot b = k mod 2:
//   copy-in stream:  [k >= 2: wait kernel(k-2)]  x[k] -> in[b]          record in_done[b]
//   caller stream:   wait in_done[b]  [k >= 2: wait out_done[b]]  kernel in[b] -> out[b]
//                                                                         record ran[b]
//   copy-out stream: wait ran[b]  out[b] -> y[k]                         record out_done[b]
// The helper streams first wait for earlier work on the caller's stream, and the caller's stream
// finally waits for the last copy back: synchronising it means every row of y is written.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <mutex>

#include "common.cuh"
#include "launch.h"

namespace nb200 {
namespace {

constexpr int kMaxDevices = 64;
constexpr int64_t kAlign = 256;
constexpr int64_t kDefaultChunkBytes = 16ll << 20;  // chunk size when the caller passes chunk_rows = 0

// Per-device helper streams and events, created on first use and kept for the process.
struct Pipe {
    cudaStream_t in = nullptr, out = nullptr;
    cudaEvent_t start = nullptr, in_done[2] = {}, ran[2] = {}, out_done[2] = {};
    bool ready = false;
};
std::mutex g_pipe_mutex[kMaxDevices];
Pipe g_pipe[kMaxDevices];

int64_t round_up(int64_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

bool float_dtype(int d) { return d == NB200_F32 || d == NB200_BF16 || d == NB200_F16; }

int make_pipe(Pipe& p) {
    if (p.ready) return NB200_OK;
    bool ok = cudaStreamCreateWithFlags(&p.in, cudaStreamNonBlocking) == cudaSuccess &&
              cudaStreamCreateWithFlags(&p.out, cudaStreamNonBlocking) == cudaSuccess &&
              cudaEventCreateWithFlags(&p.start, cudaEventDisableTiming) == cudaSuccess;
    for (int b = 0; ok && b < 2; ++b)
        ok = cudaEventCreateWithFlags(&p.in_done[b], cudaEventDisableTiming) == cudaSuccess &&
             cudaEventCreateWithFlags(&p.ran[b], cudaEventDisableTiming) == cudaSuccess &&
             cudaEventCreateWithFlags(&p.out_done[b], cudaEventDisableTiming) == cudaSuccess;
    if (!ok) {
        set_error("nb200_rms_norm_host: cannot create the copy streams: %s", cudaGetErrorString(cudaGetLastError()));
        return NB200_ERR_LAUNCH;
    }
    p.ready = true;
    return NB200_OK;
}

int64_t chunk_rows_for(int64_t rows, int64_t row_bytes, int64_t chunk_rows) {
    if (chunk_rows <= 0) chunk_rows = kDefaultChunkBytes / row_bytes;
    if (chunk_rows < 1) chunk_rows = 1;
    return chunk_rows < rows ? chunk_rows : rows;
}

// Rows of chunk k (the k-th from the start) when `remaining` rows are left, with at most c rows per
// chunk: the first chunks ramp up (c/8, c/4, c/2) so the first copy back starts early, and the
// last ones halve down to c/8 so the last copy back is short. Both ends of the pipeline then cost
// a fraction of a full chunk's transfer.
int64_t ramp_rows(int64_t k, int64_t remaining, int64_t c) {
    int64_t n = k < 3 ? c >> (3 - k) : c;
    const int64_t tail = (remaining + 1) / 2;
    if (n > tail) n = tail;
    const int64_t floor_rows = c / 8 > 0 ? c / 8 : 1;
    if (n < floor_rows) n = floor_rows;
    return n < remaining ? n : remaining;
}

}  // namespace
}  // namespace nb200

using namespace nb200;

extern "C" {

int64_t nb200_rms_norm_host_work_bytes(int dtype, int64_t ncols, int64_t chunk_rows) {
    if (!float_dtype(dtype) || ncols <= 0 || chunk_rows < 0) return -1;
    const int64_t row_bytes = ncols * (int64_t)dtype_size(dtype);
    if (chunk_rows == 0) chunk_rows = chunk_rows_for(INT64_MAX, row_bytes, 0);
    return round_up(row_bytes) + 4 * round_up(chunk_rows * row_bytes);
}

int nb200_rms_norm_host(const void* x, const void* gamma, int dtype, int64_t rows, int64_t ncols, double eps,
                        void* y, int64_t chunk_rows, void* work, int64_t work_bytes, void* stream) {
    if (!float_dtype(dtype)) {
        set_error("nb200_rms_norm_host: unsupported dtype %d; expected float16/bfloat16/float32", dtype);
        return NB200_ERR_ARG;
    }
    if (rows < 0 || ncols <= 0 || chunk_rows < 0) {
        set_error("nb200_rms_norm_host: needs rows >= 0, ncols > 0, chunk_rows >= 0");
        return NB200_ERR_ARG;
    }
    if (!std::isfinite(eps) || eps <= 0) {
        set_error("RMSNorm requires an explicit finite positive eps");
        return NB200_ERR_ARG;
    }
    if (rows == 0) return NB200_OK;
    if (!x || !gamma || !y || !work) {
        set_error("nb200_rms_norm_host: null pointer");
        return NB200_ERR_ARG;
    }
    const int64_t row_bytes = ncols * (int64_t)dtype_size(dtype);
    const int64_t crows = chunk_rows_for(rows, row_bytes, chunk_rows);
    const int64_t need = round_up(row_bytes) + 4 * round_up(crows * row_bytes);
    if (reinterpret_cast<uintptr_t>(work) % kAlign != 0 || work_bytes < need) {
        set_error("nb200_rms_norm_host: work must be %lld-byte aligned and hold %lld bytes (got %lld)",
                  (long long)kAlign, (long long)need, (long long)work_bytes);
        return NB200_ERR_ARG;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        set_error("nb200_rms_norm_host: no usable current CUDA device");
        return NB200_ERR_LAUNCH;
    }
    std::lock_guard<std::mutex> lock(g_pipe_mutex[dev]);
    Pipe& p = g_pipe[dev];
    int rc = make_pipe(p);
    if (rc) return rc;

    const cudaStream_t st = (cudaStream_t)stream;
    uint8_t* base = static_cast<uint8_t*>(work);
    uint8_t* gd = base;
    uint8_t* in[2] = {base + round_up(row_bytes), base + round_up(row_bytes) + round_up(crows * row_bytes)};
    uint8_t* out[2] = {in[1] + round_up(crows * row_bytes), in[1] + 2 * round_up(crows * row_bytes)};
    const uint8_t* xh = static_cast<const uint8_t*>(x);
    uint8_t* yh = static_cast<uint8_t*>(y);

    cudaError_t e = cudaEventRecord(p.start, st);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(p.in, p.start, 0);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(p.out, p.start, 0);
    if (e == cudaSuccess) e = cudaMemcpyAsync(gd, gamma, row_bytes, cudaMemcpyHostToDevice, p.in);
    int64_t r0 = 0;
    for (int64_t k = 0; e == cudaSuccess && rc == NB200_OK && r0 < rows; ++k) {
        const int b = (int)(k & 1);
        const int64_t nr = ramp_rows(k, rows - r0, crows);
        const size_t bytes = (size_t)(nr * row_bytes);
        if (k >= 2) e = cudaStreamWaitEvent(p.in, p.ran[b], 0);
        if (e == cudaSuccess) e = cudaMemcpyAsync(in[b], xh + r0 * row_bytes, bytes, cudaMemcpyHostToDevice, p.in);
        if (e == cudaSuccess) e = cudaEventRecord(p.in_done[b], p.in);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(st, p.in_done[b], 0);
        if (e == cudaSuccess && k >= 2) e = cudaStreamWaitEvent(st, p.out_done[b], 0);
        if (e != cudaSuccess) break;
        rc = launch_rms(in[b], gd, dtype, nr, ncols, ncols, 1, 1, (float)eps, out[b], nullptr, st);
        if (rc) break;
        e = cudaEventRecord(p.ran[b], st);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(p.out, p.ran[b], 0);
        if (e == cudaSuccess) e = cudaMemcpyAsync(yh + r0 * row_bytes, out[b], bytes, cudaMemcpyDeviceToHost, p.out);
        if (e == cudaSuccess) e = cudaEventRecord(p.out_done[b], p.out);
        r0 += nr;
    }
    // Join: the caller's stream waits for the last copies in both directions, also after an
    // error, so that nothing queued here outlives what the caller's stream orders.
    const cudaError_t j1 = cudaEventRecord(p.start, p.out);
    const cudaError_t j2 = j1 == cudaSuccess ? cudaStreamWaitEvent(st, p.start, 0) : j1;
    const cudaError_t j3 = cudaEventRecord(p.in_done[0], p.in);
    const cudaError_t j4 = j3 == cudaSuccess ? cudaStreamWaitEvent(st, p.in_done[0], 0) : j3;
    if (rc) return rc;
    if (e == cudaSuccess) e = j2 != cudaSuccess ? j2 : j4;
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error("nb200_rms_norm_host: %s", cudaGetErrorString(e));
        return NB200_ERR_LAUNCH;
    }
    return NB200_OK;
}

}  // extern "C"
