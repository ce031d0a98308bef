// W8A8 GEMM on CUDA cores for small token counts (decode micro-batches of a few tokens).
//
// y[m, n] = dequant( sum_k xq[m, k] * w[n, k] ), int8 x int8 -> int32 via dp4a.
// The weight stream dominates (1 byte per weight, read once per launch), so the kernel is
// laid out for HBM: each warp owns R output rows, its lanes split K into 16-byte vectors
// (a warp reads 512 contiguous bytes of a row per step), every lane accumulates MT tokens
// for its R rows, and a warp shuffle reduction finishes the dot products. Token codes are
// re-read through L1 (they are tiny and shared by every warp of the SM). Integer sums are
// exact, so the reduction order does not matter.
#include "common.cuh"

namespace s8b {
namespace {

constexpr int kGemvWarps = 8;
constexpr int kGemvRows = 4;  // output rows per warp

__device__ __forceinline__ int dot16(const int4 a, const int4 b, int acc) {
  acc = __dp4a(a.x, b.x, acc);
  acc = __dp4a(a.y, b.y, acc);
  acc = __dp4a(a.z, b.z, acc);
  acc = __dp4a(a.w, b.w, acc);
  return acc;
}

template <typename T, int MT>
__global__ void __launch_bounds__(kGemvWarps * 32)
    gemv_w8a8_kernel(const int8_t *__restrict__ xq, const float *__restrict__ xs,
                     const int8_t *__restrict__ w, const float *__restrict__ ws,
                     void *__restrict__ y, int out_kind, int M, int N, int K, int m0) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int n0 = (blockIdx.x * kGemvWarps + warp) * kGemvRows;
  if (n0 >= N) return;
  const int kv = K >> 4;  // 16-byte vectors per row
  const int4 *wv = reinterpret_cast<const int4 *>(w);
  const int4 *xv = reinterpret_cast<const int4 *>(xq);
  int acc[kGemvRows][MT];
#pragma unroll
  for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
    for (int t = 0; t < MT; ++t) acc[r][t] = 0;

  for (int k = lane; k < kv; k += 32) {
    int4 wr[kGemvRows];
#pragma unroll
    for (int r = 0; r < kGemvRows; ++r) {
      const int n = min(n0 + r, N - 1);
      wr[r] = __ldcs(wv + static_cast<size_t>(n) * kv + k);
    }
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      const int m = min(m0 + t, M - 1);
      const int4 xr = __ldg(xv + static_cast<size_t>(m) * kv + k);
#pragma unroll
      for (int r = 0; r < kGemvRows; ++r) acc[r][t] = dot16(wr[r], xr, acc[r][t]);
    }
  }
#pragma unroll
  for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
    for (int t = 0; t < MT; ++t) acc[r][t] = warp_sum_i(acc[r][t]);

  // Lane (r*MT + t) % 32 writes output (m0+t, n0+r).
#pragma unroll
  for (int r = 0; r < kGemvRows; ++r) {
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      if (((r * MT + t) & 31) != lane) continue;
      const int n = n0 + r, m = m0 + t;
      if (n >= N || m >= M) continue;
      const size_t o = static_cast<size_t>(m) * N + n;
      if (out_kind == 1) {
        static_cast<int32_t *>(y)[o] = acc[r][t];
      } else {
        const float v = __fmul_rn(__fmul_rn(static_cast<float>(acc[r][t]), xs[m]), ws[n]);
        static_cast<T *>(y)[o] = from_f32<T>(v);
      }
    }
  }
}

template <typename T>
int launch_gemv(const int8_t *xq, const float *xs, const int8_t *w, const float *ws, void *y,
                int out_kind, int M, int N, int K, cudaStream_t st) {
  const int rows_per_block = kGemvWarps * kGemvRows;
  const dim3 grid((N + rows_per_block - 1) / rows_per_block);
  // Token tiles of 8, then 4, 2, 1 for the remainder (the weight stream is re-read per tile;
  // the tensor-core path takes over for large token counts).
  int launches = 0;
  for (int m0 = 0; m0 < M; ++launches) {
    const int mt = M - m0;
    const int b = kGemvWarps * 32;
    if (mt >= 8) {
      gemv_w8a8_kernel<T, 8><<<grid, b, 0, st>>>(xq, xs, w, ws, y, out_kind, M, N, K, m0);
      m0 += 8;
    } else if (mt >= 4) {
      gemv_w8a8_kernel<T, 4><<<grid, b, 0, st>>>(xq, xs, w, ws, y, out_kind, M, N, K, m0);
      m0 += 4;
    } else if (mt >= 2) {
      gemv_w8a8_kernel<T, 2><<<grid, b, 0, st>>>(xq, xs, w, ws, y, out_kind, M, N, K, m0);
      m0 += 2;
    } else {
      gemv_w8a8_kernel<T, 1><<<grid, b, 0, st>>>(xq, xs, w, ws, y, out_kind, M, N, K, m0);
      m0 += 1;
    }
  }
  return check_launch(launches);
}

}  // namespace
}  // namespace s8b

using namespace s8b;

extern "C" int s8b_gemm_w8a8(const int8_t *xq, const float *xs, const int8_t *w, const float *ws,
                             void *y, int out_kind, int M, int N, int K, int dtype, void *stream) {
  if (!xq || !w || !y || (out_kind == 0 && (!xs || !ws))) return S8B_ERR_ARG;
  if (M < 0 || N <= 0 || K <= 0 || K % 16 != 0) return S8B_ERR_SHAPE;
  if (out_kind != 0 && out_kind != 1) return S8B_ERR_ARG;
  if (!aligned(xq, 16) || !aligned(w, 16)) return S8B_ERR_ALIGN;
  if (M == 0) return S8B_OK;
  S8B_DISPATCH_DTYPE(dtype, T,
                     return launch_gemv<T>(xq, xs, w, ws, y, out_kind, M, N, K,
                                           (cudaStream_t)stream));
}
