// Row-wide totals over a cluster of CTAs (row kernels and the attention row merge).
#pragma once

#include "common.cuh"

namespace s8b {
namespace {

// Row-wide totals over a cluster of CL CTAs that split one row, by pushing: each CTA stores
// its block total into slot `rank` of every CTA's array with st.async, which completes on
// that CTA's mbarrier as a byte count, and then waits on its own mbarrier until all CL values
// are in; every CTA reduces its array in rank order (the same order in every CTA). One
// one-way transfer per reduction instead of a cluster barrier, and since no CTA reads a
// peer's shared memory, none has to wait for its peers before it exits. The only cluster
// barrier (the peers' mbarriers must be initialised before anything is sent) is split:
// arrive at kernel entry, wait just before the first send, so the row loads hide it.
constexpr int kMaxRowCluster = 4;
struct ClusterRed {
  uint64_t bar[2];  // [0]: double totals, [1]: float maxima (each used once per launch)
  double d[kMaxRowCluster];
  float f[kMaxRowCluster];
};
__device__ __forceinline__ uint32_t dsmem_addr(const void *p, int rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
               : "=r"(r)
               : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))), "r"(rank));
  return r;
}
template <int CL>
__device__ __forceinline__ void cred_init(ClusterRed *r) {
  if (CL == 1) return;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(
          static_cast<uint32_t>(__cvta_generic_to_shared(&r->bar[i]))));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
template <int CL>
__device__ __forceinline__ void cred_ready() {
  if (CL > 1) asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Sends `bits` (the value's 8 or 4 bytes) to every CTA's slot and waits (bounded) for this
// CTA's CL slots. Returns false on timeout (the caller poisons its output).
template <int CL, int BYTES>
__device__ __forceinline__ bool cred_exchange(uint64_t bits, void *slots, uint64_t *bar, int rank) {
  const uint32_t lbar = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(lbar), "r"(CL * BYTES)
                 : "memory");
#pragma unroll
    for (int q = 0; q < CL; ++q) {
      const uint32_t dst = dsmem_addr(static_cast<uint8_t *>(slots) + rank * BYTES, q);
      const uint32_t rb = dsmem_addr(bar, q);
      if (BYTES == 8)
        asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b64 [%0], %1, [%2];" ::"r"(dst),
                     "l"(bits), "r"(rb)
                     : "memory");
      else
        asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(dst),
                     "r"(static_cast<uint32_t>(bits)), "r"(rb)
                     : "memory");
    }
  }
  uint64_t t0 = 0;
  for (int it = 0;; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], 0;\n"
        "selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(lbar)
        : "memory");
    if (ok) return true;
    uint64_t now;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
    if (it == 0) t0 = now;
    if (now - t0 > 100000000ull) return false;  // 100 ms: a peer never sent
  }
}
template <int CL>
__device__ __forceinline__ double cluster_total_d(double v, ClusterRed *r, int rank, bool *ok) {
  if (CL == 1) return v;
  *ok = cred_exchange<CL, 8>(static_cast<uint64_t>(__double_as_longlong(v)), r->d, &r->bar[0], rank) && *ok;
  double t = 0.0;
#pragma unroll
  for (int q = 0; q < CL; ++q) t += r->d[q];
  return t;
}
template <int CL>
__device__ __forceinline__ float cluster_max(float v, ClusterRed *r, int rank, bool *ok) {
  if (CL == 1) return v;
  *ok = cred_exchange<CL, 4>(static_cast<uint64_t>(__float_as_uint(v)), r->f, &r->bar[1], rank) && *ok;
  float t = 0.0f;
#pragma unroll
  for (int q = 0; q < CL; ++q) t = fmaxf(t, r->f[q]);
  return t;
}
template <int CL>
__device__ __forceinline__ int cluster_rank_of() {
  if (CL == 1) return 0;
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return static_cast<int>(r);
}

}  // namespace
}  // namespace s8b
