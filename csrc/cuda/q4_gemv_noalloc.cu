// Allocation-free C entry point of the dense 4-bit decode GEMV (declared in
// syn/gemv_noalloc.h).  This entry point has no counterpart in the reference project.
//
// Who needs it: callers that cannot allocate device memory at call time.  A plain C/C++
// serving loop that links this library without torch has no caching allocator to borrow a
// workspace from, and cudaMalloc/cudaFree there would synchronise the device in the middle
// of a decode step and can fail under memory pressure after the KV cache has claimed the
// rest of HBM.  Such a caller gets the whole split-K workspace from a fixed array in the
// module's device image instead.
#include <cuda_runtime.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "syn/gemv_noalloc.h"
#include "syn/launch.h"

namespace {

constexpr size_t kWsBytes = (size_t)SYN_NOALLOC_WS_FLOATS * sizeof(float);
constexpr size_t kCtrBytes = (size_t)(SYN_NOALLOC_MAX_N / 64) * sizeof(unsigned);
constexpr size_t kTableBytes = 256;  // qw pointer, sm pointer, token offsets [0, rows]
constexpr size_t kScratchBytes = kWsBytes + kCtrBytes + kTableBytes;
constexpr int kMaxDevices = 64;

// One scratch array per device (the module is loaded once per device context).  It keeps
// the contents of the previous call; the set-up kernel below clears what must start at zero.
static __device__ __align__(256) unsigned char g_gemv_scratch[kScratchBytes];

std::mutex g_addr_mu;
void* g_addr[kMaxDevices] = {};

// Writes the one-entry pointer tables and token offsets the GEMV reads, and zeroes the
// arrival counters of the split-K reduction (n_ctr of them).
__global__ void noalloc_setup_kernel(unsigned char* base, const void* qw, const void* sm, int rows, int n_ctr) {
  unsigned* ctr = reinterpret_cast<unsigned*>(base + kWsBytes);
  for (int i = threadIdx.x; i < n_ctr; i += blockDim.x) ctr[i] = 0u;
  if (threadIdx.x == 0) {
    int64_t* tab = reinterpret_cast<int64_t*>(base + kWsBytes + kCtrBytes);
    tab[0] = reinterpret_cast<int64_t>(qw);
    tab[1] = reinterpret_cast<int64_t>(sm);
    int32_t* off = reinterpret_cast<int32_t*>(tab + 2);
    off[0] = 0;
    off[1] = rows;
  }
}

int fail(char* err, int err_len, int code, const char* msg) {
  if (err && err_len > 0) snprintf(err, (size_t)err_len, "syn_q4_gemv_dense_noalloc: %s", msg);
  return code;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int syn_q4_gemv_dense_noalloc(
    const void* x, int rows, int ldx, const void* qw, const void* sm, void* out, int N, int K, int mode,
    cudaStream_t stream, char* err, int err_len) {
  if (!x || !qw || !sm || !out) return fail(err, err_len, -1, "null pointer argument");
  if (rows < 1 || rows > 64) return fail(err, err_len, -1, "rows must be in 1..64");
  if (K <= 0 || N <= 0 || K % 128 || N % 64)
    return fail(err, err_len, -1, "N must be a positive multiple of 64 and K of 128");
  if (ldx < K || (ldx * 2) % 16 || (reinterpret_cast<uintptr_t>(x) & 15))
    return fail(err, err_len, -1, "x rows must be 16-byte aligned with ldx >= K");
  if (mode != 0 && mode != 1 && mode != 3 && mode != 5) return fail(err, err_len, -1, "mode must be 0, 1, 3 or 5");
  if (N > SYN_NOALLOC_MAX_N) {
    char m[160];
    snprintf(m, sizeof(m), "N=%d exceeds the scratch limit of %d rows", N, SYN_NOALLOC_MAX_N);
    return fail(err, err_len, -1, m);
  }
  // the split the launcher will use must fit the fixed scratch: plan with the same
  // 8-row-rounded token count the launcher plans with (a.nt_hint * 8 below)
  const int nt_hint = (rows + 7) / 8;
  const int plan_rows = nt_hint * 8 < 64 ? nt_hint * 8 : 64;
  int nt = 0, kr = 0;
  size_t need = 0;
  if (!syn::q4_gemv_dense_plan(N, K, plan_rows, &nt, &kr, &need))
    return fail(err, err_len, -1, "unsupported shape: K must be a multiple of 128");
  if (need > SYN_NOALLOC_WS_FLOATS) {
    char m[200];
    snprintf(m, sizeof(m), "N=%d, K=%d, rows=%d needs %zu workspace floats; the fixed scratch holds %u", N, K, rows,
             need, (unsigned)SYN_NOALLOC_WS_FLOATS);
    return fail(err, err_len, -1, m);
  }

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(err, err_len, (int)e, cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(err, err_len, -1, "device ordinal out of range");
  unsigned char* base = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_addr_mu);
    if (!g_addr[dev]) {
      // once per device, with that device current (before any stream capture begins)
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_gemv_scratch);
      if (e != cudaSuccess) return fail(err, err_len, (int)e, cudaGetErrorString(e));
      g_addr[dev] = p;
    }
    base = static_cast<unsigned char*>(g_addr[dev]);
  }

  noalloc_setup_kernel<<<1, 256, 0, stream>>>(base, qw, sm, rows, N / 64);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(err, err_len, (int)e, cudaGetErrorString(e));

  syn::GemvArgs a;
  memset(&a, 0, sizeof(a));
  int64_t* tab = reinterpret_cast<int64_t*>(base + kWsBytes + kCtrBytes);
  a.x = x;
  a.qw_ptrs = tab;
  a.sm_ptrs = tab + 1;
  a.tok_off = reinterpret_cast<const int32_t*>(tab + 2);
  a.out = out;
  a.N = N;
  a.K = K;
  a.ldx = ldx;
  a.mode = mode;
  a.E = 1;
  a.nt_hint = nt_hint;
  e = syn::launch_q4_gemv_dense(a, reinterpret_cast<float*>(base), reinterpret_cast<unsigned*>(base + kWsBytes),
                                (size_t)SYN_NOALLOC_WS_FLOATS, stream);
  if (e != cudaSuccess) return fail(err, err_len, (int)e, cudaGetErrorString(e));
  return 0;
}
