// Allocation-free local MoE token permutation: one extern "C" entry point.
//
// This entry point has no counterpart in the reference. It exists for callers that
// cannot allocate GPU memory at the time they call us: code running inside a custom
// allocator or memory-pool callback, runtimes that pre-plan every byte of device memory
// up front and forbid allocation afterwards, and plain C / FFI hosts that have no
// PyTorch caching allocator to borrow from. Such callers own their inputs and outputs
// and pass them in; every temporary buffer this function needs lives in one fixed-size
// `static __device__` array inside the library, reserved when the library's device
// code is loaded on a GPU (and held by every GPU that loads it until the process exits).
//
// What it computes: on ONE GPU holding all E experts, the expert-grouped layout of the
// tokens' top-k copies, exactly as the expert-parallel dispatch does for world size 1:
//   xp[p]        token row of the p-th (token, choice) in expert-major order; every
//                expert group starts at a multiple of 64 rows and its padding rows are
//                zero-filled (group_off[g] .. group_off[g+1])
//   group_off    [E + 1] row offset of every expert group (group_off[E] = rows used)
//   row_w[p]     gate weight of the copy placed at row p (0 on padding rows)
//   row_src[p]   token index of the copy at row p (-1 on padding rows)
//   inv_rows     [T, k] row of each (token, choice) in xp (-1 if dropped)
//   status       [1] int32 device word, set to 0 by the call; afterwards 3 if the rows
//                did not fit cap_rows, or 5 if some expert id in topk_e was >= E or
//                < -1 (corrupted routing; those choices are dropped)
//
// Expert ids: an id of -1 means "not routed": that choice is skipped silently (it gets
// inv_rows = -1 and no row), which is how callers mask out choices. Ids >= E or < -1 are
// also skipped, with inv_rows = -1, and additionally set status to 5.
//
// Limits (compile-time, the scratch array is sized for them):
//   T <= 8192 tokens, 1 <= k <= 8, E <= 256 experts, H a multiple of 8,
//   cap_rows >= T * k + 64 * E.
// Larger sizes are rejected before anything is launched.
//
// Return value: 0 on success; 1 T out of range; 2 k out of range; 3 E out of range;
// 4 bad H; 5 cap_rows too small; 6 null pointer; 7 the scratch address could not be
// obtained on the current device; 8 x or xp not 16-byte aligned (rows move as 16-byte
// vectors); 9 a CUDA error from earlier, unrelated work was already pending on the
// calling thread (it is left pending for the caller's own checks and nothing is
// launched); 100 + cudaError_t for a launch failure of this call. A one-line message is
// also printed to stderr for every non-zero return.
//
// Set-up: the first call on each device (with that device current) looks up the
// scratch array's device address with cudaGetSymbolAddress and caches it, keyed by the
// device's current context (after a cudaDeviceReset the next call looks it up again).
// Make that first call before any CUDA stream capture begins on the device.
//
// Concurrency: all calls on a device share the one scratch array, and it keeps the last
// call's contents. Calls that may run at the same time on the GPU (different streams
// without ordering between them) race on it; order them on one stream or with events.
#pragma once
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

__attribute__((visibility("default"))) int sepx_moe_permute_noalloc(const void* x, const int* topk_e, const float* topk_w, int T, int k, int H,
                             int E, void* xp, int cap_rows, int* group_off, float* row_w, int* row_src,
                             int* inv_rows, int* status, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
