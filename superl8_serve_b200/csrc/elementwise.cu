// Row kernels of the decode step: activation quantization, fused residual + RMSNorm + quant,
// SwiGLU + quant, embedding gather, greedy argmax. One CTA per token row; these kernels move
// a few KB per token and exist to keep the int8 GEMMs fed with per-token codes.
#include "common.cuh"

namespace s8b {

namespace {

constexpr int kRowThreads = 256;

// -------------------------------------------------------------------------- quant_rows ----
template <typename T>
__global__ void __launch_bounds__(kRowThreads) quant_rows_kernel(const T *__restrict__ x,
                                                                 int8_t *__restrict__ q,
                                                                 float *__restrict__ s, int K) {
  __shared__ float red[32];
  const int m = blockIdx.x;
  const T *xr = x + static_cast<size_t>(m) * K;
  float amax = 0.0f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) amax = fmaxf(amax, fabsf(to_f32(xr[k])));
  amax = block_max(amax, red);
  const QParams p = qparams(amax, 127.0f);
  int8_t *qr = q + static_cast<size_t>(m) * K;
  for (int k = threadIdx.x; k < K; k += blockDim.x) qr[k] = static_cast<int8_t>(qcode(to_f32(xr[k]), p.inv, 127));
  if (threadIdx.x == 0) s[m] = p.scale;
}

// ---------------------------------------------------------------------- rmsnorm_quant ----
// x = h (+ residual) rounded to T, y = T((x * r) * w), codes of y. x is kept in shared
// memory (binary32) between the passes.
template <typename T>
__global__ void __launch_bounds__(kRowThreads)
    rmsnorm_quant_kernel(const T *__restrict__ h, const T *__restrict__ res_in,
                         T *__restrict__ res_out, const T *__restrict__ w, float eps,
                         int8_t *__restrict__ q, float *__restrict__ s, T *__restrict__ y_out,
                         int H) {
  extern __shared__ float xs[];
  __shared__ double redd[32];
  __shared__ float red[32];
  const int m = blockIdx.x;
  const size_t off = static_cast<size_t>(m) * H;
  double ss = 0.0;
  for (int k = threadIdx.x; k < H; k += blockDim.x) {
    float x = to_f32(h[off + k]);
    if (res_in) x = round_to<T>(__fadd_rn(x, to_f32(res_in[off + k])));
    if (res_out) res_out[off + k] = from_f32<T>(x);
    xs[k] = x;
    ss += static_cast<double>(x) * static_cast<double>(x);
  }
  ss = block_sum_d(ss, redd);
  const float r = rms_factor(ss, H, eps);
  float amax = 0.0f;
  for (int k = threadIdx.x; k < H; k += blockDim.x) {
    const float y = round_to<T>(__fmul_rn(__fmul_rn(xs[k], r), to_f32(w[k])));
    xs[k] = y;
    amax = fmaxf(amax, fabsf(y));
  }
  amax = block_max(amax, red);
  const QParams p = qparams(amax, 127.0f);
  for (int k = threadIdx.x; k < H; k += blockDim.x) {
    const float y = xs[k];
    q[off + k] = static_cast<int8_t>(qcode(y, p.inv, 127));
    if (y_out) y_out[off + k] = from_f32<T>(y);
  }
  if (threadIdx.x == 0) s[m] = p.scale;
}

// ---------------------------------------------------------------------- silu_mul_quant ----
template <typename T>
__global__ void __launch_bounds__(kRowThreads)
    silu_mul_quant_kernel(const T *__restrict__ gu, int F, T *__restrict__ y_out,
                          int8_t *__restrict__ q, float *__restrict__ s) {
  extern __shared__ float ys[];
  __shared__ float red[32];
  const int m = blockIdx.x;
  const T *row = gu + static_cast<size_t>(m) * 2 * F;
  float amax = 0.0f;
  for (int k = threadIdx.x; k < F; k += blockDim.x) {
    const float g = to_f32(row[k]);
    const float u = to_f32(row[F + k]);
    const float a = round_to<T>(__fdiv_rn(g, __fadd_rn(1.0f, exp_s8b(-g))));
    const float y = round_to<T>(__fmul_rn(a, u));
    ys[k] = y;
    amax = fmaxf(amax, fabsf(y));
  }
  amax = block_max(amax, red);
  const QParams p = qparams(amax, 127.0f);
  const size_t off = static_cast<size_t>(m) * F;
  for (int k = threadIdx.x; k < F; k += blockDim.x) {
    q[off + k] = static_cast<int8_t>(qcode(ys[k], p.inv, 127));
    if (y_out) y_out[off + k] = from_f32<T>(ys[k]);
  }
  if (threadIdx.x == 0) s[m] = p.scale;
}

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

template <typename T>
__global__ void __launch_bounds__(kRowThreads) argmax_kernel(const T *__restrict__ logits, int V,
                                                             int32_t *__restrict__ out) {
  __shared__ float sv[32];
  __shared__ int si[32];
  const int m = blockIdx.x;
  const T *row = logits + static_cast<size_t>(m) * V;
  float bv = -__int_as_float(0x7f800000);
  int bi = 0x7fffffff;
  for (int k = threadIdx.x; k < V; k += blockDim.x) better(bv, bi, to_f32(row[k]), k);
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
    if (lane == 0) out[m] = bi;
  }
}

}  // namespace

}  // namespace s8b

using namespace s8b;

extern "C" int s8b_quant_rows(const void *x, int dtype, int8_t *q, float *s, int M, int K,
                              void *stream) {
  if (!x || !q || !s) return S8B_ERR_ARG;
  if (M < 0 || K <= 0) return S8B_ERR_SHAPE;
  if (M == 0) return S8B_OK;
  S8B_DISPATCH_DTYPE(dtype, T,
                     quant_rows_kernel<T><<<M, kRowThreads, 0, (cudaStream_t)stream>>>(
                         static_cast<const T *>(x), q, s, K));
  return check_launch();
}

extern "C" int s8b_rmsnorm_quant(const void *h, const void *residual_in, void *residual_out,
                                 const void *w, float eps, int8_t *q, float *s, void *y_out,
                                 int M, int H, int dtype, void *stream) {
  if (!h || !w || !q || !s) return S8B_ERR_ARG;
  if (M < 0 || H <= 0 || H > 16384) return S8B_ERR_SHAPE;
  if (M == 0) return S8B_OK;
  const size_t smem = static_cast<size_t>(H) * sizeof(float);
  S8B_DISPATCH_DTYPE(dtype, T, {
    auto kern = rmsnorm_quant_kernel<T>;
    ensure_smem(reinterpret_cast<const void *>(kern), smem);
    kern<<<M, kRowThreads, smem, (cudaStream_t)stream>>>(
        static_cast<const T *>(h), static_cast<const T *>(residual_in),
        static_cast<T *>(residual_out), static_cast<const T *>(w), eps, q, s,
        static_cast<T *>(y_out), H);
  });
  return check_launch();
}

extern "C" int s8b_silu_mul_quant(const void *gu, int M, int F, void *y_out, int8_t *q, float *s,
                                  int dtype, void *stream) {
  if (!gu || !q || !s) return S8B_ERR_ARG;
  if (M < 0 || F <= 0 || F > 49152) return S8B_ERR_SHAPE;
  if (M == 0) return S8B_OK;
  const size_t smem = static_cast<size_t>(F) * sizeof(float);
  S8B_DISPATCH_DTYPE(dtype, T, {
    auto kern = silu_mul_quant_kernel<T>;
    ensure_smem(reinterpret_cast<const void *>(kern), smem);
    kern<<<M, kRowThreads, smem, (cudaStream_t)stream>>>(static_cast<const T *>(gu), F,
                                                        static_cast<T *>(y_out), q, s);
  });
  return check_launch();
}

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
                     argmax_kernel<T><<<M, kRowThreads, 0, (cudaStream_t)stream>>>(
                         static_cast<const T *>(logits), V, out));
  return check_launch();
}
