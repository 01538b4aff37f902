// Allocation-free C entry point of the dense 4-bit decode GEMV.
//
// This entry point has no counterpart in the reference project.
//
// It runs the same split-K kernel as the torch op `q4_gemv_dense`, but takes its split-K
// workspace, arrival counters and one-entry pointer tables from a fixed scratch array that
// lives in the module's device image, so a call allocates no device or host memory.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// Scratch limits: split-K partial sums of at most SYN_NOALLOC_WS_FLOATS floats
// (16 MiB) and at most SYN_NOALLOC_MAX_N output rows of the weight matrix.
#define SYN_NOALLOC_WS_FLOATS (4u << 20)
#define SYN_NOALLOC_MAX_N 262144

// out = x @ W^T for one 4-bit weight matrix in the tiled device layout (qw/sm as written by
// q4_quantize / q4_rows_to_tiled).  x: bf16 [rows, ldx] with rows in 1..64, K % 128 == 0,
// N % 64 == 0, 16-byte aligned rows.  mode: 0 bf16 store [rows, N]; 1 SwiGLU of
// interleaved gate/up rows, bf16 [rows, N/2]; 3 f32 accumulate into out [rows, N];
// 5 f32 store [rows, N].  Work is queued on `stream`.
//
// Returns 0 on success; a cudaError_t value (> 0) from the CUDA runtime; or -1 for an
// argument or size this entry point rejects.  When err/err_len are given, a one-line
// message is written there on failure.
//
// The first call on a device looks up the scratch address with cudaGetSymbolAddress while
// that device is current; make that first call before any stream capture begins.  The
// scratch is shared by every call on a device: calls that overlap in time (two streams,
// two host threads) race on it and must be serialised by the caller.  The looked-up address
// is kept per device ordinal for the life of the process: after cudaDeviceReset (which
// unloads the module and creates a new primary context on next use) it is stale, so a
// process that resets a device must not call this entry point on it again.
int syn_q4_gemv_dense_noalloc(const void* x, int rows, int ldx, const void* qw, const void* sm, void* out,
                              int N, int K, int mode, cudaStream_t stream, char* err, int err_len);

#ifdef __cplusplus
}
#endif
