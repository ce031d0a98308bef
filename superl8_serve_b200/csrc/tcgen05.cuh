// tcgen05 / TMA / mbarrier building blocks shared by the tensor-core kernels (sm_100a).
// Every wait is bounded (mbar_wait gives up after `limit_ns`, raising a CTA abort flag and a
// global status word) so no kernel can hang on a barrier that never completes.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include <map>
#include <mutex>

#include "common.cuh"

namespace s8b {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait. Returns false (and raises the CTA abort flag and the global status) on timeout
// or when another role of the CTA already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort,
                                          int32_t *status,
                                          unsigned long long limit_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = now_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (now_ns() - t0 > limit_ns) {
      *abort = 1;
      atomicExch(status, S8B_ERR_TIMEOUT);
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, int c0, int c1,
                                            int c2, int c3, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

// Bounded wait that ignores the abort flag: used on the way out of an aborted kernel, to let
// copies already in flight land before the CTA's shared memory is released.
__device__ __forceinline__ bool mbar_drain(uint64_t *bar, uint32_t parity,
                                           unsigned long long limit_ns = 100000000ull) {
  const uint64_t t0 = now_ns();
  while (!mbar_try_wait(bar, parity))
    if (now_ns() - t0 > limit_ns) return false;
  return true;
}

// Named barrier over `n` threads that also returns, to all of them, whether any passed `p`.
__device__ __forceinline__ bool group_any(int id, int n, bool p) {
  uint32_t r;
  asm volatile(
      "{\n.reg .pred a, b;\nsetp.ne.u32 a, %1, 0;\nbar.red.or.pred b, %2, %3, a;\n"
      "selp.u32 %0, 1, 0, b;\n}\n"
      : "=r"(r)
      : "r"(p ? 1u : 0u), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void group_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// Plain bulk copy global -> shared of `bytes` contiguous bytes (16-byte aligned, multiple of
// 16), completing on the stage's mbarrier like a TMA tile load.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes,
                                          uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor, K-major operand in 128B-swizzled 8-row x 128-byte atoms:
// start >> 4 in [0,14), SBO = 1024 B (stride between 8-row groups) in [32,46), descriptor
// version 1 in [46,48), layout SWIZZLE_128B (2) in [61,64). LBO is unused for this layout.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>(1) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor kind::i8: D s32 [4,6)=2, A/B format (s8 = 1, u8 = 0) in [7,10) /
// [10,13), A/B major (0 = K, 1 = MN) bits 15/16, N>>3 in [17,23), M>>4 in [24,29).
__host__ __device__ constexpr uint32_t i8_idesc(int M, int N, bool a_signed = true,
                                                 bool b_signed = true, bool a_mn_major = false,
                                                 bool b_mn_major = false) {
  return (2u << 4) | ((a_signed ? 1u : 0u) << 7) | ((b_signed ? 1u : 0u) << 10) |
         ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(
          tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z));
}
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t addr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(addr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void epi_bar_sync(int nthreads = 128) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}


// ------------------------------------------------------------------- host helpers ----
inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void *p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D uint8 tensor map with 128B swizzle: `outer` rows of `inner` bytes, `pitch` bytes apart;
// one copy moves a box of box_inner bytes x box_outer rows.
inline int make_map_2d(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer,
                       uint64_t pitch, uint32_t box_inner, uint32_t box_outer) {
  auto fn = encode_fn();
  if (!fn) return S8B_ERR_CUDA;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {pitch};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? S8B_OK : S8B_ERR_ALIGN;
}

// 4-D tiled map over a paged KV pool laid out [blocks][heads][rows][128 B] (dims innermost
// first: 128 bytes, rows per block, heads, blocks), box {128, rows, 1, nb}: one head's rows of
// nb consecutive blocks, landing in block order with the same 128B swizzle as the 2-D row maps.
inline int make_map_kv4(CUtensorMap *map, const void *base, uint32_t rows, uint32_t heads,
                        uint64_t nblocks, uint32_t nb) {
  auto fn = encode_fn();
  if (!fn) return S8B_ERR_CUDA;
  const cuuint64_t dims[4] = {128, rows, heads, nblocks};
  const cuuint64_t strides[3] = {128, 128ull * rows, 128ull * rows * heads};
  const cuuint32_t box[4] = {128, rows, 1, nb};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void *>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? S8B_OK : S8B_ERR_ALIGN;
}

// Bytes from `p` to the end of the device allocation that contains it (0 if unknown): the
// extent a tensor map over a caller's buffer may cover.
inline size_t bytes_to_alloc_end(const void *p) {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void *f = nullptr;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(f);
  });
  if (!fn) return 0;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(p)) != CUDA_SUCCESS) return 0;
  const uint64_t a = reinterpret_cast<uint64_t>(p);
  return a >= base && a < base + size ? static_cast<size_t>(base + size - a) : 0;
}

inline int sm_count() {
  static std::mutex mu;
  static std::map<int, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  cache[dev] = n > 0 ? n : 148;
  return cache[dev];
}

}  // namespace tc
}  // namespace s8b
