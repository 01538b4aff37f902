// Router-predicted expert prefetch for decode.  The routing kernel of layer i also ranks the
// experts of layer i+1 (its router rows applied to layer i's hidden state) and emits a
// prediction mask.  This kernel, launched on a side stream right after that routing, copies
// the predicted experts of layer i+1 that live in the pinned host tier into a VRAM staging
// bank (zero-copy reads over PCIe, a few CTAs so the main stream keeps the rest of the GPU)
// and rewrites layer i+1's per-expert pointer tables: predicted host experts -> their staging
// rows, every other expert -> its home pointer.  Layer i+1's GEMVs wait on the side stream
// (event) and then stream the prefetched experts from HBM; mispredicted host experts are
// still read in place.  Reference: RFC-0023 §9 / RFC-0040 :998 (router predicts the next
// layer's experts so host->VRAM expert transfers overlap the current layer).
#include "common.cuh"

namespace syn {

struct PrefetchPart {
  const uint8_t* host;      // host-tier rows (pinned, device-mapped)
  uint8_t* stage;           // staging rows in VRAM (same row order)
  int64_t row_bytes;        // bytes per expert row (multiple of 16)
  int64_t* live;            // [El] pointer table read by the GEMV
  const int64_t* home;      // [El] home pointers (VRAM slot or host row)
};

struct PrefetchArgs {
  const int32_t* pred;      // [E global] 1 = predicted for the next layer
  const int32_t* host_row;  // [El] host row of a host-tier expert, -1 if resident
  int e0, El, chunks;
  PrefetchPart part[4];     // (gate_up q, gate_up scales, down q, down scales)
  int n_parts;
};

__global__ void __launch_bounds__(256) expert_prefetch_kernel(PrefetchArgs a) {
  // pointer tables first (CTA 0): consistent with the copies below once the side stream ends
  if (blockIdx.x == 0) {
    for (int e = threadIdx.x; e < a.El; e += blockDim.x) {
      const int h = a.host_row[e];
      const bool take = h >= 0 && a.pred[a.e0 + e] != 0;
      for (int p = 0; p < a.n_parts; ++p) {
        const PrefetchPart& P = a.part[p];
        P.live[e] = take ? reinterpret_cast<int64_t>(P.stage + (int64_t)h * P.row_bytes) : P.home[e];
      }
    }
  }
  // copies: work item = (expert, chunk of each part's row)
  for (int w = blockIdx.x; w < a.El * a.chunks; w += gridDim.x) {
    const int e = w / a.chunks, c = w % a.chunks;
    const int h = a.host_row[e];
    if (h < 0 || a.pred[a.e0 + e] == 0) continue;
    for (int p = 0; p < a.n_parts; ++p) {
      const PrefetchPart& P = a.part[p];
      const int64_t nvec = P.row_bytes / 16;
      const int64_t per = (nvec + a.chunks - 1) / a.chunks;
      const int64_t v0 = c * per, v1 = min(nvec, v0 + per);
      const uint4* src = reinterpret_cast<const uint4*>(P.host + (int64_t)h * P.row_bytes);
      uint4* dst = reinterpret_cast<uint4*>(P.stage + (int64_t)h * P.row_bytes);
      // four 16-byte reads in flight per thread: PCIe latency needs many outstanding requests
      int64_t v = v0 + threadIdx.x;
      for (; v + 3 * blockDim.x < v1; v += 4 * blockDim.x) {
        const uint4 r0 = __ldcs(src + v), r1 = __ldcs(src + v + blockDim.x);
        const uint4 r2 = __ldcs(src + v + 2 * blockDim.x), r3 = __ldcs(src + v + 3 * blockDim.x);
        dst[v] = r0;
        dst[v + blockDim.x] = r1;
        dst[v + 2 * blockDim.x] = r2;
        dst[v + 3 * blockDim.x] = r3;
      }
      for (; v < v1; v += blockDim.x) dst[v] = __ldcs(src + v);
    }
  }
}

cudaError_t launch_expert_prefetch(const int32_t* pred, const int32_t* host_row, int e0, int El,
                                   const void* const* host, void* const* stage, const int64_t* row_bytes,
                                   int64_t* const* live, const int64_t* const* home, int n_parts, int ctas,
                                   cudaStream_t s) {
  if (n_parts < 1 || n_parts > 4 || El <= 0) return cudaErrorInvalidValue;
  PrefetchArgs a;
  a.pred = pred;
  a.host_row = host_row;
  a.e0 = e0;
  a.El = El;
  a.chunks = 8;
  a.n_parts = n_parts;
  for (int p = 0; p < n_parts; ++p) {
    if (row_bytes[p] % 16) return cudaErrorInvalidValue;
    a.part[p] = PrefetchPart{reinterpret_cast<const uint8_t*>(host[p]), reinterpret_cast<uint8_t*>(stage[p]),
                             row_bytes[p], live[p], home[p]};
  }
  expert_prefetch_kernel<<<ctas, 256, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace syn
