// Small runtime kernels of the step graph (reference op list: crates/kernels/src/op/kind.rs):
//  * doorbells: a bounded device wait on a 32-bit flag (the stream-wait role; never an
//    unbounded spin: after the limit it sets an error bit and returns) and a release store;
//  * `Timestamp`: one %globaltimer sample into a buffer slot (profiled graph variants);
//  * `TapGather` / `HiddenTap`: copy selected rows of a hidden state to an f32 tap buffer and
//    compare two tap buffers on the device (parity checks against an oracle);
//  * `KvPack` / `KvUnpack`: gather the K/V pages of a block list into one contiguous buffer
//    (for host offload or migration) and scatter them back.
#include "common.cuh"
#include "sync.cuh"

namespace syn {

__device__ __forceinline__ float tap_f32(float v) { return v; }
__device__ __forceinline__ float tap_f32(__nv_bfloat16 v) { return bf2f(v); }

__global__ void doorbell_wait_kernel(const uint32_t* flag, uint32_t want, uint64_t timeout_ns, int* status,
                                     uint64_t* waited_ns) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const uint64_t t0 = globaltimer_ns();
  wait_flag(flag, want, timeout_ns, status, 0);
  if (waited_ns) *waited_ns = globaltimer_ns() - t0;
}

__global__ void doorbell_ring_kernel(uint32_t* flag, uint32_t value) {
  if (threadIdx.x == 0 && blockIdx.x == 0) st_release_sys(flag, value);
}

__global__ void timestamp_kernel(uint64_t* out, int slot) {
  if (threadIdx.x == 0 && blockIdx.x == 0) out[slot] = globaltimer_ns();
}

// rows idx[i] of src (bf16 or f32, [R, H]) -> dst f32 [n, H]
template <typename T>
__global__ void tap_gather_kernel(const T* __restrict__ src, const int32_t* __restrict__ idx, int H,
                                  float* __restrict__ dst) {
  const int i = blockIdx.x;
  const int64_t r = idx[i];
  for (int c = threadIdx.x; c < H; c += blockDim.x) dst[(int64_t)i * H + c] = tap_f32(src[r * H + c]);
}

// per row: max |a - b| and ||a - b|| / ||b||  -> out [n, 2]
__global__ void tap_compare_kernel(const float* __restrict__ a, const float* __restrict__ b, int H,
                                   float* __restrict__ out) {
  const int i = blockIdx.x;
  float mx = 0.f, d2 = 0.f, b2 = 0.f;
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    const float x = a[(int64_t)i * H + c], y = b[(int64_t)i * H + c];
    mx = fmaxf(mx, fabsf(x - y));
    d2 += (x - y) * (x - y);
    b2 += y * y;
  }
  __shared__ float red[32];
  mx = block_max(mx, red);
  d2 = block_sum(d2, red);
  b2 = block_sum(b2, red);
  if (threadIdx.x == 0) {
    out[i * 2] = mx;
    out[i * 2 + 1] = sqrtf(d2) / fmaxf(sqrtf(b2), 1e-30f);
  }
}

// page p = pages[i]: K and V rows [Hkv, 16, D] of that page <-> packed[i][2][Hkv*16*D]
template <bool PACK>
__global__ void kv_pages_kernel(uint4* __restrict__ kc, uint4* __restrict__ vc, const int32_t* __restrict__ pages,
                                int page_vec, uint4* __restrict__ packed) {
  const int i = blockIdx.y;
  const int64_t p = pages[i];
  for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < page_vec; v += gridDim.x * blockDim.x) {
    uint4* pk = packed + ((int64_t)i * 2) * page_vec + v;
    uint4* pv = pk + page_vec;
    if (PACK) {
      *pk = kc[p * page_vec + v];
      *pv = vc[p * page_vec + v];
    } else {
      kc[p * page_vec + v] = *pk;
      vc[p * page_vec + v] = *pv;
    }
  }
}

cudaError_t launch_doorbell_wait(const uint32_t* flag, uint32_t want, uint64_t timeout_ns, int* status,
                                 uint64_t* waited_ns, cudaStream_t s) {
  doorbell_wait_kernel<<<1, 32, 0, s>>>(flag, want, timeout_ns, status, waited_ns);
  return cudaGetLastError();
}

cudaError_t launch_doorbell_ring(uint32_t* flag, uint32_t value, cudaStream_t s) {
  doorbell_ring_kernel<<<1, 32, 0, s>>>(flag, value);
  return cudaGetLastError();
}

cudaError_t launch_timestamp(uint64_t* out, int slot, cudaStream_t s) {
  timestamp_kernel<<<1, 32, 0, s>>>(out, slot);
  return cudaGetLastError();
}

cudaError_t launch_tap_gather(const void* src, bool src_bf16, const int32_t* idx, int n, int H, float* dst,
                              cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  if (src_bf16)
    tap_gather_kernel<__nv_bfloat16><<<n, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(src), idx, H, dst);
  else
    tap_gather_kernel<float><<<n, 256, 0, s>>>(reinterpret_cast<const float*>(src), idx, H, dst);
  return cudaGetLastError();
}

cudaError_t launch_tap_compare(const float* a, const float* b, int n, int H, float* out, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  tap_compare_kernel<<<n, 256, 0, s>>>(a, b, H, out);
  return cudaGetLastError();
}

cudaError_t launch_kv_pages(void* kc, void* vc, const int32_t* pages, int n, int64_t page_bytes, void* packed,
                            bool pack, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  if (page_bytes % 16) return cudaErrorInvalidValue;
  const int page_vec = (int)(page_bytes / 16);
  dim3 grid((unsigned)((page_vec + 255) / 256), (unsigned)n);
  if (pack)
    kv_pages_kernel<true><<<grid, 256, 0, s>>>(reinterpret_cast<uint4*>(kc), reinterpret_cast<uint4*>(vc), pages,
                                               page_vec, reinterpret_cast<uint4*>(packed));
  else
    kv_pages_kernel<false><<<grid, 256, 0, s>>>(reinterpret_cast<uint4*>(kc), reinterpret_cast<uint4*>(vc), pages,
                                                page_vec, reinterpret_cast<uint4*>(packed));
  return cudaGetLastError();
}

}  // namespace syn
