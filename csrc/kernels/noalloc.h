// Allocation-free sum of squares: tn5b_grad_sqsum_noalloc
//
// This entry point has no counterpart in the TempName-5090 reference; it is an
// addition of this library.
//
// Who it is for: callers that cannot allocate device memory.  A plugin or
// custom-op host that owns every byte of device memory under a fixed budget
// does not let the code it hosts call cudaMalloc, and cudaMalloc / cudaFree
// synchronise the whole device, which a latency-critical loop cannot afford.
// The regular entry point (grad_sqsum, via the Python bindings) takes a
// caller-allocated workspace tensor for its per-block partial sums; this
// variant keeps those partials in a fixed array that is part of the loaded
// library instead, so the caller passes only its input and its output.
//
// Contract:
//   int tn5b_grad_sqsum_noalloc(const void* grad, int grad_is_fp32, int64_t n,
//                               double* out, void* stream);
//   *out = sum over i < n of float(grad[i])^2, accumulated in double, computed
//   in a fixed order (the result does not depend on the GPU model or timing).
//   grad: device array of n BF16 (grad_is_fp32 == 0) or FP32 values, 16-byte
//   aligned; n > 0 and a multiple of 8.  out: one device double.  stream: a
//   cudaStream_t (may be null for the legacy default stream).
//   Returns 0 on success (launches are asynchronous on `stream`),
//   -1 for an invalid argument, -2 when n exceeds the maximum below (nothing
//   is launched), or a positive cudaError_t from set-up or launch.
//
// Limit: the scratch is a file-scope __device__ array of 16384 doubles
// (128 KiB).  Every GPU that loads the library holds it until the process
// exits.  Each 16384-element chunk of the input produces one partial, so n is
// at most 16384 * 16384 = 268,435,456 elements per call.
//
// Set-up: the first call on each device, with that device current, looks up
// the device address of the array with cudaGetSymbolAddress (host code cannot
// use the array's name as a device pointer).  Make that first call before any
// stream capture on the device.  No call allocates memory: no cudaMalloc,
// cudaFree or allocating library routine is used.
//
// Sharing: every call on a device uses the same array, which keeps the last
// call's contents.  Each call writes every partial it later reads, so nothing
// has to start at zero.  Calls whose kernels overlap on the GPU (different
// streams without ordering between them) race on the array; order them.
#pragma once
#include <cstdint>

extern "C" __attribute__((visibility("default"))) int tn5b_grad_sqsum_noalloc(
    const void* grad, int grad_is_fp32, int64_t n, double* out,
                                       void* stream);
