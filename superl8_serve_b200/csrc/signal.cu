// Stage-to-stage signalling over NVLink without host involvement.
//
// A flag is a uint32 in device memory, usually a peer's (the consumer owns it, the producer
// writes it across NVLink). Values compared are "epochs" that increase by one per decode
// step; they live in device memory so a captured CUDA graph replays with fresh values.
// Every wait is bounded: after the timeout the waiting kernel records S8B_ERR_TIMEOUT and
// the awaited value in a status word and returns, so no stream can hang on a missing peer.
#include "common.cuh"

namespace s8b {
namespace {

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__global__ void flag_set_kernel(uint32_t *flag, const uint32_t *value, uint32_t add) {
  __threadfence_system();
  st_release_sys(flag, *value + add);
}

__global__ void flag_wait_kernel(const uint32_t *flag, const uint32_t *value, uint32_t add,
                                 uint64_t timeout_ns, int32_t *status) {
  const uint32_t want = *value + add;
  const uint64_t t0 = globaltimer();
  while (true) {
    const uint32_t v = ld_acquire_sys(flag);
    if (static_cast<int32_t>(v - want) >= 0) break;
    if (globaltimer() - t0 > timeout_ns) {
      if (status) {
        status[1] = static_cast<int32_t>(want);
        status[2] = static_cast<int32_t>(v);
        atomicExch(status, S8B_ERR_TIMEOUT);
      }
      return;
    }
    __nanosleep(64);
  }
  __threadfence_system();
}

__global__ void counter_add_kernel(uint32_t *ctr, uint32_t inc) { *ctr += inc; }

// Copies a short list of buffers (usually into a peer's memory over NVLink) with plain
// stores from one CTA, then raises `flag` like flag_set_kernel: every thread's stores are
// ordered before the release by the CTA barrier and thread 0's system-scope fence.
constexpr int kPutMax = 8;
struct PutList {
  void *dst[kPutMax];
  const void *src[kPutMax];
  unsigned long long bytes[kPutMax];
  int n;
};

__global__ void __launch_bounds__(1024)
    peer_put_flag_kernel(PutList L, uint32_t *flag, const uint32_t *value, uint32_t add) {
  for (int i = 0; i < L.n; ++i) {
    const unsigned long long nb = L.bytes[i];
    const uintptr_t d = reinterpret_cast<uintptr_t>(L.dst[i]);
    const uintptr_t sa = reinterpret_cast<uintptr_t>(L.src[i]);
    if (((d | sa | nb) & 15) == 0) {
      const int4 *sp = static_cast<const int4 *>(L.src[i]);
      int4 *dp = static_cast<int4 *>(L.dst[i]);
      for (unsigned long long k = threadIdx.x; k < nb / 16; k += blockDim.x) dp[k] = sp[k];
    } else if (((d | sa | nb) & 3) == 0) {
      const uint32_t *sp = static_cast<const uint32_t *>(L.src[i]);
      uint32_t *dp = static_cast<uint32_t *>(L.dst[i]);
      for (unsigned long long k = threadIdx.x; k < nb / 4; k += blockDim.x) dp[k] = sp[k];
    } else {
      const uint8_t *sp = static_cast<const uint8_t *>(L.src[i]);
      uint8_t *dp = static_cast<uint8_t *>(L.dst[i]);
      for (unsigned long long k = threadIdx.x; k < nb; k += blockDim.x) dp[k] = sp[k];
    }
  }
  if (flag == nullptr) return;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    st_release_sys(flag, *value + add);
  }
}

__global__ void advance_kernel(int32_t *positions, int32_t *context_lens, int M, int inc) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < M) {
    const int p = positions[i] + inc;
    positions[i] = p;
    if (context_lens) context_lens[i] = p + 1;
  }
}

}  // namespace
}  // namespace s8b

using namespace s8b;

extern "C" int s8b_flag_set(uint32_t *flag, const uint32_t *value, uint32_t add, void *stream) {
  if (!flag || !value) return S8B_ERR_ARG;
  flag_set_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(flag, value, add);
  return check_launch();
}

extern "C" int s8b_flag_wait(const uint32_t *flag, const uint32_t *value, uint32_t add,
                             uint64_t timeout_ns, int32_t *status, void *stream) {
  if (!flag || !value) return S8B_ERR_ARG;
  flag_wait_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(flag, value, add, timeout_ns, status);
  return check_launch();
}

extern "C" int s8b_peer_put_flag(void *const *dst, const void *const *src, const size_t *bytes,
                                 int n, uint32_t *flag, const uint32_t *value, uint32_t add,
                                 void *stream) {
  if (n < 0 || n > kPutMax) return S8B_ERR_SHAPE;
  if ((n > 0 && (!dst || !src || !bytes)) || (flag && !value)) return S8B_ERR_ARG;
  PutList L{};
  L.n = n;
  for (int i = 0; i < n; ++i) {
    if (bytes[i] > 0 && (!dst[i] || !src[i])) return S8B_ERR_ARG;
    L.dst[i] = dst[i];
    L.src[i] = src[i];
    L.bytes[i] = bytes[i];
  }
  peer_put_flag_kernel<<<1, 1024, 0, (cudaStream_t)stream>>>(L, flag, value, add);
  return check_launch();
}

extern "C" int s8b_counter_add(uint32_t *ctr, uint32_t inc, void *stream) {
  if (!ctr) return S8B_ERR_ARG;
  counter_add_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(ctr, inc);
  return check_launch();
}

extern "C" int s8b_advance(int32_t *positions, int32_t *context_lens, int M, int inc,
                           void *stream) {
  if (!positions) return S8B_ERR_ARG;
  if (M < 0) return S8B_ERR_SHAPE;
  if (M == 0) return S8B_OK;
  advance_kernel<<<(M + 127) / 128, 128, 0, (cudaStream_t)stream>>>(positions, context_lens, M, inc);
  return check_launch();
}

extern "C" int s8b_flag_status(const int32_t *status_host_copy) {
  if (!status_host_copy) return S8B_ERR_ARG;
  return status_host_copy[0];
}
