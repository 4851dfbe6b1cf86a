// Router top-K selection for callers that may not allocate device memory.
//
// Some callers cannot call cudaMalloc (or any allocator) on the path that
// launches this work: an inference server plugin whose host framework owns and
// pre-plans every byte of device memory and forbids allocation while work is
// enqueued, or a caller reaching this library through an FFI with no device
// allocator of its own.  For them ossa_router_topk_noalloc runs the same
// selection as ossa_router_topk but takes its workspace from a fixed array in
// device memory that belongs to this library.
//
// The array is a file-scope __device__ variable: every GPU that loads the
// library holds its kNoAllocScratchBytes until the process exits.  Its name is
// only a host-side stand-in, so the device address is looked up with
// cudaGetSymbolAddress, with the device current: the first call on each device
// does the lookup (make that first call before any stream capture), and every
// later call made while its stream is not capturing looks it up again, so a
// context torn down and created again (cudaDeviceReset) cannot leave a stale
// address behind.  Calls made during a capture use the address of the last
// lookup.  The stream must belong to the current device.  All calls share the
// one array: calls whose work overlaps on the GPU (different streams, or
// different host threads) race on it and must be serialised by the caller.  The
// array keeps the previous call's contents; ossa_router_topk clears the parts
// that must start at zero on every call.  Its first 8 bytes are the counters of
// the last call (rows sent to the exact fallback, status word), which
// ossa_router_status_noalloc reads.
#include "../../include/ossa_b200.h"
#include "kernels.h"

#include <cuda_runtime.h>
#include <mutex>
#include <stdio.h>

namespace {

constexpr size_t kNoAllocScratchBytes = 32ull << 20;  // 32 MiB

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_lock;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device: looked up on the
// first call and on every call whose stream is not capturing; a capturing
// stream reuses the last address (a lookup is not a stream operation, but the
// capture should record exactly what the caller enqueues).
cudaError_t scratch_address(cudaStream_t stream, void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    e = cudaStreamIsCapturing(stream, &cap);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> guard(g_lock);
    if (!g_scratch_ptr[dev] || cap == cudaStreamCaptureStatusNone) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return cudaSuccess;
}

}  // namespace

extern "C" {

int ossa_router_topk_noalloc(const void* q, const void* k, int dtype, const float* wq, const float* wk,
                                      const float* pos_bias, int B, int H, int Hkv, int N, int D, int r,
                                      int seq_len_cfg, int K, int causal, int32_t* idx_out,
                                      ossa_stream_t stream) {
    const size_t need = ossa_router_workspace_size(B, H, Hkv, N, r, K);
    char msg[256];
    if (need > kNoAllocScratchBytes) {
        snprintf(msg, sizeof(msg),
                 "ossa_router_topk_noalloc: this shape needs %zu bytes of workspace, more than the %zu-byte "
                 "built-in scratch; use ossa_router_topk with a caller-provided workspace",
                 need, kNoAllocScratchBytes);
        ossa::set_error_message(msg);
        return OSSA_ERR_WORKSPACE;
    }
    void* ws = nullptr;
    const cudaError_t e = scratch_address(static_cast<cudaStream_t>(stream), &ws);
    if (e != cudaSuccess) {
        snprintf(msg, sizeof(msg), "ossa_router_topk_noalloc: scratch address lookup failed: %s",
                 cudaGetErrorString(e));
        ossa::set_error_message(msg);
        return OSSA_ERR_CUDA;
    }
    return ossa_router_topk(q, k, dtype, wq, wk, pos_bias, B, H, Hkv, N, D, r, seq_len_cfg, K, causal, idx_out,
                            ws, kNoAllocScratchBytes, stream);
}

int ossa_router_status_noalloc(int* fallback_rows, int* status) {
    int h[2] = {0, 0};
    // synchronous read of the counters block at the start of this device's array
    const cudaError_t e = cudaMemcpyFromSymbol(h, g_noalloc_scratch, sizeof(h), 0, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) {
        char msg[256];
        snprintf(msg, sizeof(msg), "ossa_router_status_noalloc: counters read failed: %s", cudaGetErrorString(e));
        ossa::set_error_message(msg);
        return OSSA_ERR_CUDA;
    }
    if (fallback_rows) *fallback_rows = h[0];
    if (status) *status = h[1];
    return OSSA_OK;
}

}  // extern "C"
