// Per-token row kernels with the whole row in registers: fused residual + RMSNorm + int8
// quantization, SwiGLU + int8 quantization, and plain int8 quantization.
//
// One CTA per token row with up to 1024 threads; each thread owns VPT vectors of 4 elements
// (8-byte loads), so a 4096-wide row is one load per thread and the row never round-trips
// through shared memory. The arithmetic per element is exactly that of the oracle
// (binary32, no contraction); only the reductions are block-wide (max is exact, the sum of
// squares accumulates in float64).
#include "cluster.cuh"
#include "common.cuh"

namespace s8b {
namespace {

template <typename T>
struct Vec4 {
  uint2 raw;
  __device__ __forceinline__ void load(const T *p) { raw = *reinterpret_cast<const uint2 *>(p); }
  __device__ __forceinline__ void store(T *p) const { *reinterpret_cast<uint2 *>(p) = raw; }
  __device__ __forceinline__ float get(int i) const {
    const unsigned short b = static_cast<unsigned short>(
        i < 2 ? (raw.x >> (16 * i)) & 0xffff : (raw.y >> (16 * (i - 2))) & 0xffff);
    T v;
    memcpy(&v, &b, 2);
    return to_f32(v);
  }
  __device__ __forceinline__ void set(int i, float f) {
    const T v = from_f32<T>(f);
    unsigned short b;
    memcpy(&b, &v, 2);
    if (i < 2)
      raw.x = (raw.x & ~(0xffffu << (16 * i))) | (static_cast<unsigned>(b) << (16 * i));
    else
      raw.y = (raw.y & ~(0xffffu << (16 * (i - 2)))) | (static_cast<unsigned>(b) << (16 * (i - 2)));
  }
};

__device__ __forceinline__ void store_codes(int8_t *dst, const float v[4], float inv) {
  char4 c;
  c.x = static_cast<signed char>(qcode(v[0], inv, 127));
  c.y = static_cast<signed char>(qcode(v[1], inv, 127));
  c.z = static_cast<signed char>(qcode(v[2], inv, 127));
  c.w = static_cast<signed char>(qcode(v[3], inv, 127));
  *reinterpret_cast<char4 *>(dst) = c;
}

template <typename T, int VPT, int CL = 1, typename Src = RowSrc<T>>
__global__ void __launch_bounds__(1024)
    rmsnorm_quant_v(Src h, const T *__restrict__ res_in, T *__restrict__ res_out,
                    const T *__restrict__ w, float eps, int8_t *__restrict__ q,
                    float *__restrict__ s, T *__restrict__ y_out, int H) {
  griddep_launch();  // the next kernel may start its prologue
  __shared__ double redd[32];
  __shared__ float red[32];
  __shared__ ClusterRed cr;
  cred_init<CL>(&cr);
  griddep_wait();    // launched with programmatic serialization
  // CL CTAs split the row: this CTA owns vectors [rank * nvec, (rank + 1) * nvec).
  const int m = blockIdx.x / CL, rank = cluster_rank_of<CL>(), nvec = (H >> 2) / CL;
  bool ok = true;
  const size_t off = static_cast<size_t>(m) * H;
  float x[VPT][4], xr[VPT][4], wg[VPT][4];
  double ss = 0.0;
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int i = rank * nvec + threadIdx.x + v * blockDim.x;
    if (threadIdx.x + v * blockDim.x < nvec) {
      Vec4<T> wv;
      wv.load(w + 4 * i);  // independent of the reduction: in flight with the row loads
      float hv[4];
      h.load4(m, 4 * i, hv);
      if constexpr (Src::kCodec) {  // the previous stage's payload: [hidden | residual]
        float rv[4];
        h.load4(m, H + 4 * i, rv);
#pragma unroll
        for (int j = 0; j < 4; ++j) x[v][j] = round_to<T>(__fadd_rn(hv[j], rv[j]));
      } else if (res_in) {
        Vec4<T> r;
        r.load(res_in + off + 4 * i);
#pragma unroll
        for (int j = 0; j < 4; ++j) x[v][j] = round_to<T>(__fadd_rn(hv[j], r.get(j)));
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) x[v][j] = hv[j];
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        xr[v][j] = x[v][j];
        wg[v][j] = wv.get(j);
        ss += static_cast<double>(x[v][j]) * static_cast<double>(x[v][j]);
      }
    }
  }
  ss = block_sum_d(ss, redd);
  cred_ready<CL>();
  ss = cluster_total_d<CL>(ss, &cr, rank, &ok);
  const float rf = rms_factor(ss, H, eps);
  float amax = 0.0f;
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    if (threadIdx.x + v * blockDim.x < nvec) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        x[v][j] = round_to<T>(__fmul_rn(__fmul_rn(x[v][j], rf), wg[v][j]));
        amax = fmaxf(amax, fabsf(x[v][j]));
      }
    }
  }
  amax = cluster_max<CL>(block_max(amax, red), &cr, rank, &ok);
  const QParams p = qparams(ok ? amax : __int_as_float(0x7fffffff), 127.0f);  // timeout: NaN scale
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int i = rank * nvec + threadIdx.x + v * blockDim.x;
    if (threadIdx.x + v * blockDim.x < nvec) {
      if (res_out) {
        Vec4<T> a;
#pragma unroll
        for (int j = 0; j < 4; ++j) a.set(j, xr[v][j]);
        a.store(res_out + off + 4 * i);
      }
      store_codes(q + off + 4 * i, x[v], p.inv);
      if (y_out) {
        Vec4<T> yv;
#pragma unroll
        for (int j = 0; j < 4; ++j) yv.set(j, x[v][j]);
        yv.store(y_out + off + 4 * i);
      }
    }
  }
  if (threadIdx.x == 0 && rank == 0) s[m] = p.scale;
}

template <typename T, int VPT, int CL = 1>
__global__ void __launch_bounds__(1024)
    silu_mul_quant_v(RowSrc<T> gu, int F, T *__restrict__ y_out, int8_t *__restrict__ q,
                     float *__restrict__ s) {
  griddep_launch();  // the next kernel may start its prologue
  __shared__ float red[32];
  __shared__ ClusterRed cr;
  cred_init<CL>(&cr);
  griddep_wait();    // launched with programmatic serialization
  const int m = blockIdx.x / CL, rank = cluster_rank_of<CL>(), nvec = (F >> 2) / CL;
  bool ok = true;
  float y[VPT][4];
  float amax = 0.0f;
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int i = rank * nvec + threadIdx.x + v * blockDim.x;
    if (threadIdx.x + v * blockDim.x < nvec) {
      float g[4], u[4];
      gu.load4(m, 4 * i, g);
      gu.load4(m, F + 4 * i, u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float gf = g[j];
        const float a = round_to<T>(__fdiv_rn(gf, __fadd_rn(1.0f, exp_s8b(-gf))));
        y[v][j] = round_to<T>(__fmul_rn(a, u[j]));
        amax = fmaxf(amax, fabsf(y[v][j]));
      }
    }
  }
  amax = block_max(amax, red);
  cred_ready<CL>();
  amax = cluster_max<CL>(amax, &cr, rank, &ok);
  const QParams p = qparams(ok ? amax : __int_as_float(0x7fffffff), 127.0f);  // timeout: NaN scale
  const size_t off = static_cast<size_t>(m) * F;
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int i = rank * nvec + threadIdx.x + v * blockDim.x;
    if (threadIdx.x + v * blockDim.x < nvec) {
      store_codes(q + off + 4 * i, y[v], p.inv);
      if (y_out) {
        Vec4<T> yv;
#pragma unroll
        for (int j = 0; j < 4; ++j) yv.set(j, y[v][j]);
        yv.store(y_out + off + 4 * i);
      }
    }
  }
  if (threadIdx.x == 0 && rank == 0) s[m] = p.scale;
}

template <typename T, int VPT>
__global__ void __launch_bounds__(1024)
    quant_rows_v(const T *__restrict__ x, int8_t *__restrict__ q, float *__restrict__ s, int K) {
  griddep_launch();  // the next kernel may start its prologue
  griddep_wait();    // launched with programmatic serialization
  __shared__ float red[32];
  const int m = blockIdx.x, nvec = K >> 2;
  const size_t off = static_cast<size_t>(m) * K;
  float v4[VPT][4];
  float amax = 0.0f;
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int i = threadIdx.x + v * blockDim.x;
    if (i < nvec) {
      Vec4<T> a;
      a.load(x + off + 4 * i);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v4[v][j] = a.get(j);
        amax = fmaxf(amax, fabsf(v4[v][j]));
      }
    }
  }
  amax = block_max(amax, red);
  const QParams p = qparams(amax, 127.0f);
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int i = threadIdx.x + v * blockDim.x;
    if (i < nvec) store_codes(q + off + 4 * i, v4[v], p.inv);
  }
  if (threadIdx.x == 0) s[m] = p.scale;
}

int row_sm_count() {
  static int n[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (n[dev] == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    n[dev] = v > 0 ? v : 148;
  }
  return n[dev];
}

// threads = nvec rounded up to a warp (at most 1024), VPT = ceil(nvec / threads) <= 8, so
// each thread carries as short a chain as the row allows. When the launch has more CTAs than
// the GPU has SMs (`ctas`), threads are capped at kRowThreads: 256-thread CTAs (about 12K
// registers) fit four to an SM, so a launch of 256 CTAs (64 rows x a 4-CTA cluster) runs in
// one wave beside a resident GEMM CTA, where 768-thread CTAs fit one to an SM by registers
// and took two waves. Longer rows take more threads (up to 1024) so that VPT stays <= 8.
constexpr int kRowThreads = 256;
inline void row_shape(int nvec, int *threads, int *vpt, long ctas = 0) {
  int t = ((nvec + 31) / 32) * 32;
  if (t > kRowThreads && ctas > row_sm_count()) t = kRowThreads;
  if ((nvec + t - 1) / t > 8) t = (((nvec + 7) / 8 + 31) / 32) * 32;
  if (t > 1024) t = 1024;
  *threads = t;
  *vpt = (nvec + t - 1) / t;
}

#define S8B_VPT_SWITCH(vpt, V, ...) \
  switch (vpt) {                    \
    case 1: { constexpr int V = 1; __VA_ARGS__; break; } \
    case 2: { constexpr int V = 2; __VA_ARGS__; break; } \
    case 3: { constexpr int V = 3; __VA_ARGS__; break; } \
    case 4: { constexpr int V = 4; __VA_ARGS__; break; } \
    case 5: { constexpr int V = 5; __VA_ARGS__; break; } \
    case 6: { constexpr int V = 6; __VA_ARGS__; break; } \
    case 7: { constexpr int V = 7; __VA_ARGS__; break; } \
    case 8: { constexpr int V = 8; __VA_ARGS__; break; } \
    default: return S8B_ERR_SHAPE; \
  }

}  // namespace
}  // namespace s8b

using namespace s8b;

extern "C" int s8b_quant_rows(const void *x, int dtype, int8_t *q, float *s, int M, int K,
                              void *stream) {
  if (!x || !q || !s) return S8B_ERR_ARG;
  if (M < 0 || K <= 0 || K % 4 != 0 || K > 32768) return S8B_ERR_SHAPE;
  if (!aligned(x, 8) || !aligned(q, 4)) return S8B_ERR_ALIGN;
  if (M == 0) return S8B_OK;
  int th, vpt;
  row_shape(K / 4, &th, &vpt, M);
  S8B_DISPATCH_DTYPE(dtype, T,
                     S8B_VPT_SWITCH(vpt, V,
                                    launch_pdl(quant_rows_v<T, V>, M, th, 0, (cudaStream_t)stream,
                                               static_cast<const T *>(x), q, s, K)));
  return check_launch();
}

namespace s8b {
namespace {
// Rows of >= 128 vectors are split over a 4-CTA cluster (latency: more SMs per row, each
// CTA a quarter of the loads); shorter rows keep one CTA per row.
constexpr int kRowCluster = kMaxRowCluster;
inline int row_cluster(int nvec) { return (nvec % kRowCluster == 0 && nvec / kRowCluster >= 32) ? kRowCluster : 1; }

template <typename T, typename Src>
int launch_rms(Src src, const void *res_in, void *res_out, const void *w, float eps,
               int8_t *q, float *s, void *y_out, int M, int H, void *stream) {
  int cl = row_cluster(H / 4);
  // a codec source needs every warp on whole 128-value blocks (inverse Hadamard across a
  // warp): each CTA's share of the row a multiple of 32 four-value vectors
  if constexpr (Src::kCodec) {
    if ((H / 4 / cl) % 32 != 0) cl = 1;
  }
  int th, vpt;
  row_shape(H / 4 / cl, &th, &vpt, static_cast<long>(M) * cl);
  const cudaStream_t st = (cudaStream_t)stream;
  if (cl == 1) {
    S8B_VPT_SWITCH(vpt, V,
                   launch_pdl(rmsnorm_quant_v<T, V, 1, Src>, M, th, 0, st, src,
                              static_cast<const T *>(res_in), static_cast<T *>(res_out),
                              static_cast<const T *>(w), eps, q, s, static_cast<T *>(y_out), H));
  } else {
    S8B_VPT_SWITCH(vpt, V,
                   launch_pdl_cluster(rmsnorm_quant_v<T, V, kRowCluster, Src>, M * kRowCluster, th, 0,
                                      kRowCluster, st, src, static_cast<const T *>(res_in),
                                      static_cast<T *>(res_out), static_cast<const T *>(w), eps,
                                      q, s, static_cast<T *>(y_out), H));
  }
  return check_launch();
}

template <typename T>
int launch_silu(RowSrc<T> src, int F, void *y_out, int8_t *q, float *s, int M, void *stream) {
  const int cl = row_cluster(F / 4);
  int th, vpt;
  row_shape(F / 4 / cl, &th, &vpt, static_cast<long>(M) * cl);
  const cudaStream_t st = (cudaStream_t)stream;
  if (cl == 1) {
    S8B_VPT_SWITCH(vpt, V,
                   launch_pdl(silu_mul_quant_v<T, V, 1>, M, th, 0, st, src, F,
                              static_cast<T *>(y_out), q, s));
  } else {
    S8B_VPT_SWITCH(vpt, V,
                   launch_pdl_cluster(silu_mul_quant_v<T, V, kRowCluster>, M * kRowCluster, th, 0,
                                      kRowCluster, st, src, F, static_cast<T *>(y_out), q, s));
  }
  return check_launch();
}
}  // namespace
}  // namespace s8b

extern "C" int s8b_rmsnorm_quant(const void *h, const void *residual_in, void *residual_out,
                                 const void *w, float eps, int8_t *q, float *s, void *y_out,
                                 int M, int H, int dtype, void *stream) {
  if (!h || !w || !q || !s) return S8B_ERR_ARG;
  if (M < 0 || H <= 0 || H % 4 != 0 || H > 32768) return S8B_ERR_SHAPE;
  if (!aligned(h, 8) || !aligned(w, 8) || !aligned(q, 4) || !aligned(residual_in, 8) ||
      !aligned(residual_out, 8) || !aligned(y_out, 8))
    return S8B_ERR_ALIGN;
  if (M == 0) return S8B_OK;
  S8B_DISPATCH_DTYPE(dtype, T,
                     return launch_rms<T>(row_src<T>(h, H), residual_in, residual_out, w, eps, q,
                                          s, y_out, M, H, stream));
}

extern "C" int s8b_rmsnorm_quant_codec(const void *payload, const float *scales, int scheme,
                                       void *residual_out, const void *w, float eps, int8_t *q,
                                       float *s, int M, int H, int dtype, void *stream) {
  if (!payload || !w || !q || !s || !residual_out || (scheme != S8B_CODEC_FP16 && !scales))
    return S8B_ERR_ARG;
  if (scheme < S8B_CODEC_FP16 || scheme > S8B_CODEC_NF4) return S8B_ERR_DTYPE;
  if (M < 0 || H <= 0 || H % 128 != 0 || H > 32768) return S8B_ERR_SHAPE;
  if (!aligned(payload, 8) || !aligned(w, 8) || !aligned(q, 4) || !aligned(residual_out, 8))
    return S8B_ERR_ALIGN;
  if (M == 0) return S8B_OK;
  S8B_DISPATCH_DTYPE(dtype, T,
                     return launch_rms<T>(row_src_codec<T>(payload, scales, scheme, 2 * H),
                                          nullptr, residual_out, w, eps, q, s, nullptr, M, H,
                                          stream));
}

extern "C" int s8b_rmsnorm_quant_split(const int32_t *part, int C, const float *xs,
                                       const float *ws, const void *residual_in,
                                       void *residual_out, const void *w, float eps, int8_t *q,
                                       float *s, void *y_out, int M, int H, int dtype,
                                       void *stream) {
  if (!part || !xs || !ws || !w || !q || !s) return S8B_ERR_ARG;
  if (M < 0 || H <= 0 || H % 4 != 0 || H > 32768 || C < 1 || C > 8) return S8B_ERR_SHAPE;
  if (!aligned(part, 16) || !aligned(ws, 16) || !aligned(w, 8) || !aligned(q, 4) ||
      !aligned(residual_in, 8) || !aligned(residual_out, 8) || !aligned(y_out, 8))
    return S8B_ERR_ALIGN;
  if (M == 0) return S8B_OK;
  S8B_DISPATCH_DTYPE(dtype, T,
                     return launch_rms<T>(row_src_split<T>(part, C, xs, ws, M, H), residual_in,
                                          residual_out, w, eps, q, s, y_out, M, H, stream));
}

extern "C" int s8b_silu_mul_quant(const void *gu, int M, int F, void *y_out, int8_t *q, float *s,
                                  int dtype, void *stream) {
  if (!gu || !q || !s) return S8B_ERR_ARG;
  if (M < 0 || F <= 0 || F % 4 != 0 || F > 32768) return S8B_ERR_SHAPE;
  if (!aligned(gu, 8) || !aligned(q, 4) || !aligned(y_out, 8)) return S8B_ERR_ALIGN;
  if (M == 0) return S8B_OK;
  S8B_DISPATCH_DTYPE(dtype, T, return launch_silu<T>(row_src<T>(gu, 2 * F), F, y_out, q, s, M,
                                                     stream));
}

extern "C" int s8b_silu_mul_quant_split(const int32_t *part, int C, const float *xs,
                                        const float *ws, int M, int F, void *y_out, int8_t *q,
                                        float *s, int dtype, void *stream) {
  if (!part || !xs || !ws || !q || !s) return S8B_ERR_ARG;
  if (M < 0 || F <= 0 || F % 4 != 0 || F > 32768 || C < 1 || C > 8) return S8B_ERR_SHAPE;
  if (!aligned(part, 16) || !aligned(ws, 16) || !aligned(q, 4) || !aligned(y_out, 8))
    return S8B_ERR_ALIGN;
  if (M == 0) return S8B_OK;
  S8B_DISPATCH_DTYPE(dtype, T,
                     return launch_silu<T>(row_src_split<T>(part, C, xs, ws, M, 2 * F), F, y_out,
                                           q, s, M, stream));
}
