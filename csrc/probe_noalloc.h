// Allocation-free variant of the TeaCache probe reduction.
//
// This entry point has no counterpart in the reference: it exists for callers
// that cannot allocate device memory themselves.  Examples are a plugin that
// runs inside a host framework which owns every device allocation through its
// own pool (so a stray cudaMalloc would break its accounting or fail outright),
// a real-time or embedded host that forbids allocation after start-up, and
// code called from a context where cudaMalloc / cudaFree would serialise the
// device or are simply not available.  Such a caller passes only its inputs
// and its output; the scratch this reduction needs lives in a fixed device
// array compiled into this library.
//
//   int dfl_rel_l1_noalloc(const void* a, const void* b, long long n,
//                          float* out, cudaStream_t stream);
//
//   out[0] = sum_i |a[i] - b[i]| / sum_i |b[i]|   (a, b: n bf16 values,
//   16-byte aligned device pointers; out: one f32 on the device)
//
// Contract:
//   * It calls no cudaMalloc, cudaFree or other allocating routine (torch's
//     included).  The scratch is a static device array of
//     DFL_NOALLOC_MAX_BLOCKS * 2 + 1 floats (about 8 KB); every GPU that loads
//     the library holds that array until the process exits.
//   * The first call on a device resolves the array's device address with
//     cudaGetSymbolAddress while that device is current; make that first call
//     before any stream capture on the device.  With lazy module loading (the
//     CUDA default) that first call is also when the driver loads this
//     library's device code on the device and reserves memory for it and for
//     the static array (with CUDA_MODULE_LOADING=EAGER, when the library is
//     loaded).  "Allocates nothing" therefore holds from the second call on:
//     a caller that forbids allocation after start-up makes one call per
//     device during its start-up.
//   * The resolved address is cached per device index for the life of the
//     process, which assumes one primary context per device.  After
//     cudaDeviceReset (or anything else that destroys and re-creates the
//     context) the cached address is stale: such a caller must not use this
//     entry point again in the same process.
//   * All calls share the one array and it keeps whatever the last call left
//     there.  The entry point clears the part that must start at zero (the
//     completion ticket) on `stream` before each launch.  Calls that overlap
//     on the GPU (different streams, no ordering between them) race on the
//     array and give wrong results: order them on one stream.
//   * Limit: the reduction uses at most DFL_NOALLOC_MAX_BLOCKS thread blocks.
//     A device that would need more (over 256 SMs) is rejected with
//     DFL_NOALLOC_ERR_TOO_LARGE instead of writing past the array.  Any n fits,
//     since each block loops over its share of the input.
//
// Return codes: 0 success; DFL_NOALLOC_ERR_ALIGN (-2) misaligned a or b;
// DFL_NOALLOC_ERR_ARGS (-3) null pointer or negative n;
// DFL_NOALLOC_ERR_TOO_LARGE (-4) more blocks than the static scratch holds;
// DFL_NOALLOC_ERR_SYMBOL (-5) cudaGetSymbolAddress failed; other positive values
// are the cudaError_t of the failed CUDA call.  dfl_rel_l1_noalloc_error_string
// turns a code into a message.
#pragma once
#include <cuda_runtime_api.h>

#define DFL_NOALLOC_MAX_BLOCKS 1024
#define DFL_NOALLOC_ERR_ALIGN (-2)
#define DFL_NOALLOC_ERR_ARGS (-3)
#define DFL_NOALLOC_ERR_TOO_LARGE (-4)
#define DFL_NOALLOC_ERR_SYMBOL (-5)

#ifdef __cplusplus
extern "C" {
#endif

int dfl_rel_l1_noalloc(const void* a, const void* b, long long n, float* out, cudaStream_t stream);
const char* dfl_rel_l1_noalloc_error_string(int code);

#ifdef __cplusplus
}
#endif
