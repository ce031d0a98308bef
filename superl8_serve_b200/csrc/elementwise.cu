// Embedding gather and greedy argmax (the per-token quantizing row kernels are in rowops.cu).
#include "common.cuh"

namespace s8b {

namespace {

constexpr int kRowThreads = 256;

// ------------------------------------------------------------------------------ embed ----
__global__ void embed_kernel(const int32_t *__restrict__ ids, const uint4 *__restrict__ table,
                             int row_vecs, uint4 *__restrict__ out) {
  const int m = blockIdx.x;
  const size_t src = static_cast<size_t>(ids[m]) * row_vecs;
  const size_t dst = static_cast<size_t>(m) * row_vecs;
  for (int i = threadIdx.x; i < row_vecs; i += blockDim.x) out[dst + i] = table[src + i];
}

// ----------------------------------------------------------------------------- argmax ----
__device__ __forceinline__ void better(float &bv, int &bi, float v, int i) {
  if (v > bv || (v == bv && i < bi)) {
    bv = v;
    bi = i;
  }
}

// One CTA per row. (value, index) pairs are ordered by value, then lowest index, so the
// result does not depend on the traversal order: each thread scans 8-value vectors (16-byte
// loads, four in flight), then warp and CTA reductions merge the candidates.
constexpr int kArgmaxThreads = 1024;

__device__ __forceinline__ void reduce_best(float &bv, int &bi, float *sv, int *si) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    better(bv, bi, ov, oi);
  }
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) {
    sv[w] = bv;
    si[w] = bi;
  }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    bv = lane < nw ? sv[lane] : -__int_as_float(0x7f800000);
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      better(bv, bi, ov, oi);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kArgmaxThreads) argmax_kernel(const T *__restrict__ logits, int V,
                                                                int32_t *__restrict__ out) {
  __shared__ float sv[32];
  __shared__ int si[32];
  griddep_wait();  // launched with programmatic serialization
  const int m = blockIdx.x;
  const T *row = logits + static_cast<size_t>(m) * V;
  float bv = -__int_as_float(0x7f800000);
  int bi = 0x7fffffff;
  const bool vec = (reinterpret_cast<uintptr_t>(row) & 15) == 0;
  const int nvec = vec ? V / 8 : 0;
  const uint4 *rv = reinterpret_cast<const uint4 *>(row);
  for (int base = threadIdx.x; base < nvec; base += 4 * kArgmaxThreads) {
    uint4 x[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = base + j * kArgmaxThreads;
      if (i < nvec) x[j] = rv[i];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = base + j * kArgmaxThreads;
      if (i >= nvec) continue;
      const T *e = reinterpret_cast<const T *>(&x[j]);
#pragma unroll
      for (int k = 0; k < 8; ++k) better(bv, bi, to_f32(e[k]), 8 * i + k);
    }
  }
  for (int k = 8 * nvec + threadIdx.x; k < V; k += kArgmaxThreads) better(bv, bi, to_f32(row[k]), k);
  reduce_best(bv, bi, sv, si);
  if (threadIdx.x == 0) out[m] = bi;
}

}  // namespace

}  // namespace s8b

using namespace s8b;

extern "C" int s8b_embed(const int32_t *ids, const void *table, int M, int H, void *out, int dtype,
                         void *stream) {
  if (!ids || !table || !out) return S8B_ERR_ARG;
  if (dtype != S8B_BF16 && dtype != S8B_FP16) return S8B_ERR_DTYPE;
  if (M < 0 || H <= 0 || (H * 2) % 16 != 0) return S8B_ERR_SHAPE;
  if (!aligned(table, 16) || !aligned(out, 16)) return S8B_ERR_ALIGN;
  if (M == 0) return S8B_OK;
  embed_kernel<<<M, 128, 0, (cudaStream_t)stream>>>(ids, static_cast<const uint4 *>(table),
                                                    H * 2 / 16, static_cast<uint4 *>(out));
  return check_launch();
}

extern "C" int s8b_argmax(const void *logits, int M, int V, int32_t *out, int dtype, void *stream) {
  if (!logits || !out) return S8B_ERR_ARG;
  if (M < 0 || V <= 0) return S8B_ERR_SHAPE;
  if (M == 0) return S8B_OK;
  S8B_DISPATCH_DTYPE(dtype, T,
                     launch_pdl(argmax_kernel<T>, M, kArgmaxThreads, 0, (cudaStream_t)stream,
                         static_cast<const T *>(logits), V, out));
  return check_launch();
}

// The library's exponential (exp_s8b: the softmax, the partition merge, SiLU), elementwise,
// so that its values can be checked against the CPU definition bit for bit.
__global__ void exp_kernel(const float *__restrict__ x, float *__restrict__ y, long long n) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    y[i] = exp_s8b(x[i]);
}

extern "C" int s8b_exp_f32(const float *x, float *y, long long n, void *stream) {
  if (n < 0) return S8B_ERR_SHAPE;
  if (n == 0) return S8B_OK;
  if (!x || !y) return S8B_ERR_ARG;
  const long long blocks = (n + 255) / 256;
  exp_kernel<<<static_cast<unsigned>(blocks < 4096 ? blocks : 4096), 256, 0,
               (cudaStream_t)stream>>>(x, y, n);
  return check_launch();
}
