// Shared device helpers for the s8b kernels (sm_100a).
//
// Numerics contract: every floating-point step that feeds a stored value is a correctly
// rounded binary32 operation written with __fmul_rn / __fadd_rn / __fsub_rn / __fdiv_rn /
// __fsqrt_rn, so nvcc cannot contract it into an FMA. The CPU oracle performs the same
// operations in the same order, which makes the two bit-identical.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/s8b.h"

namespace s8b {

// --------------------------------------------------------------------- error plumbing ----
void record_cuda_error(cudaError_t e);
int check_launch(int launches = 1);  // S8B_OK or S8B_ERR_CUDA; counts kernel launches
// Raise a kernel's dynamic shared-memory limit to `bytes` on the current device, once per
// (kernel, device): the attribute call happens on the first (eager) launch, never again
// while a stream is being captured into a CUDA graph.
void ensure_smem(const void *kernel, size_t bytes);

inline bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Programmatic dependent launch: wait for the preceding kernel's results (a no-op when the
// launch carries no programmatic dependency) / let the next kernel in the stream start its
// prologue early (its own wait still covers this kernel's completion).
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void griddep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Launch with programmatic stream serialization: the kernel may start while the previous
// kernel in the stream is still running, so it must call griddep_wait() (every CTA) before
// touching global memory that earlier kernels write or read; only its prologue overlaps.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}
// The same with thread-block clusters of `cluster` CTAs along x.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                               int cluster, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// ----------------------------------------------------------------------------- dtypes ----
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
// Round a binary32 value to the activation dtype and back (exact after the first rounding).
template <typename T> __device__ __forceinline__ float round_to(float x) {
  return to_f32(from_f32<T>(x));
}

// ---------------------------------------------------------------------------- exp -----
// exp(x) by range reduction to 2^t = 2^k * 2^f (k = rint(t), |f| <= 1/2) and the degree-7
// Taylor polynomial of 2^f = sum (f ln2)^i / i!. Coefficients are the binary32 roundings of
// ln(2)^i / i!; Horner with separate multiply and add; 2^k built from its exponent bits.
// Written without branches (the out-of-range cases are selects), so that a thread's
// independent calls interleave. rint(tc) comes from adding and subtracting 1.5 * 2^23: for
// |tc| <= 127 the sum's round-to-nearest-even lands exactly on rint(tc), and k's integer value
// sits in the sum's low mantissa bits (no float-to-int conversion on the chain).
__device__ __forceinline__ float exp_s8b(float x) {
  const float t = __fmul_rn(x, 0x1.715476p+0f);  // x * log2(e)
  const float tc = fminf(fmaxf(t, -125.0f), 127.0f);  // == t wherever the result is finite
  const float kb = __fadd_rn(tc, 0x1.8p23f);
  const float k = __fsub_rn(kb, 0x1.8p23f);      // rint(tc)
  const float f = __fsub_rn(tc, k);
  float p = 0x1.ffcbfcp-17f;
  p = __fadd_rn(__fmul_rn(p, f), 0x1.430912p-13f);
  p = __fadd_rn(__fmul_rn(p, f), 0x1.5d87fep-10f);
  p = __fadd_rn(__fmul_rn(p, f), 0x1.3b2ab6p-7f);
  p = __fadd_rn(__fmul_rn(p, f), 0x1.c6b08ep-5f);
  p = __fadd_rn(__fmul_rn(p, f), 0x1.ebfbe0p-3f);
  p = __fadd_rn(__fmul_rn(p, f), 0x1.62e430p-1f);
  p = __fadd_rn(__fmul_rn(p, f), 1.0f);
  const int ki = __float_as_int(kb) - 0x4B400000;  // k as an integer, in [-125, 127]
  float r = __fmul_rn(p, __int_as_float((ki + 127) << 23));
  r = t < -125.0f ? 0.0f : r;
  r = t > 127.0f ? __int_as_float(0x7f800000) : r;
  return t != t ? t : r;  // NaN in, NaN out
}

// Warp-wide maximum in one instruction (sm_100a). NaN inputs are ignored, as with fmaxf.
__device__ __forceinline__ float warp_max_redux(float v) {
  float r;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
  return r;
}

constexpr float kHadScale = 0x1.6a09e6p-4f;  // binary32 rounding of 128^-1/2

// ------------------------------------------------------- Hadamard-128 in one warp -----
// A warp holds one 128-vector, lane l owning elements 4l..4l+3 in v[0..3]. Stage h pairs
// (j, j+h) with j's bit h clear and replaces them by (a+b, a-b). Stages 1 and 2 are inside a
// lane; stages 4..64 pair lane l with lane l ^ (h/4).
__device__ __forceinline__ void fwht128_warp(float v[4]) {
  float a, b;
  a = v[0]; b = v[1]; v[0] = __fadd_rn(a, b); v[1] = __fsub_rn(a, b);
  a = v[2]; b = v[3]; v[2] = __fadd_rn(a, b); v[3] = __fsub_rn(a, b);
  a = v[0]; b = v[2]; v[0] = __fadd_rn(a, b); v[2] = __fsub_rn(a, b);
  a = v[1]; b = v[3]; v[1] = __fadd_rn(a, b); v[3] = __fsub_rn(a, b);
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int dl = 1; dl < 32; dl <<= 1) {
    const bool lower = (lane & dl) == 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float o = __shfl_xor_sync(0xffffffffu, v[i], dl);
      v[i] = lower ? __fadd_rn(v[i], o) : __fsub_rn(o, v[i]);
    }
  }
}

// ---------------------------------------------------------------------------- NF4 --------
// The 16-entry 4-bit NormalFloat codebook (QLoRA, Dettmers et al. 2023): 8 positive and 7
// negative standard-normal quantiles at evenly spaced probabilities between 0.5 and
// 0.9677083, plus 0, normalised to [-1, 1], rounded to binary32, ascending.
__device__ constexpr float kNF4[16] = {
    -1.0f, -0.6961929202079773f, -0.5250730514526367f, -0.39491748809814453f,
    -0.28444135189056396f, -0.18477343022823334f, -0.09104999154806137f, 0.0f,
    0.07958032935857773f, 0.16093017160892487f, 0.24611228704452515f, 0.33791518211364746f,
    0.44070979952812195f, 0.5626169443130493f, 0.7229567170143127f, 1.0f};

// Codebook entry of code c (0..15) by a select tree on c's bits (no memory access).
__device__ __forceinline__ float nf4_value(int c) {
  float l[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) l[i] = (c & 1) ? kNF4[2 * i + 1] : kNF4[2 * i];
#pragma unroll
  for (int i = 0; i < 4; ++i) l[i] = (c & 2) ? l[2 * i + 1] : l[2 * i];
#pragma unroll
  for (int i = 0; i < 2; ++i) l[i] = (c & 4) ? l[2 * i + 1] : l[2 * i];
  return (c & 8) ? l[1] : l[0];
}

// Index of the entry nearest to y: argmin_i |y - kNF4[i]| in binary32, lowest i on ties.
__device__ __forceinline__ int nf4_code(float y) {
  int best = 0;
  float bd = fabsf(__fsub_rn(y, kNF4[0]));
#pragma unroll
  for (int i = 1; i < 16; ++i) {
    const float d = fabsf(__fsub_rn(y, kNF4[i]));
    if (d < bd) {
      bd = d;
      best = i;
    }
  }
  return best;
}

// ------------------------------------------------------------------------- reductions -----
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide reductions (all threads receive the result). `red` holds >= 32 elements.
__device__ __forceinline__ float block_max(float v, float *red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  v = lane < nw ? red[lane] : 0.0f;
  return warp_max(v);
}
__device__ __forceinline__ double block_sum_d(double v, double *red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum_d(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  v = lane < nw ? red[lane] : 0.0;
  return warp_sum_d(v);
}

// ------------------------------------------------------------------ row input source ----
// A row-major [M][ld] input of dtype T, or the split-K partial sums of a tensor-core GEMM
// (int32 [C][M][ld], out_kind 2) that are summed and dequantized exactly as the GEMM's own
// epilogue would: v = dtype((f32(sum_c part) * xs[m]) * ws[col]). col is a multiple of 4;
// x and part are 8- / 16-byte aligned, ws 16-byte aligned.
template <typename T>
struct RowSrc {
  const T *x;
  const int32_t *part;
  const float *xs, *ws;
  size_t cstride;  // M * ld
  int C, ld;
  static constexpr bool kCodec = false;
  __device__ __forceinline__ void load4(int m, int col, float v[4]) const {
    const size_t o = static_cast<size_t>(m) * ld + col;
    if (part == nullptr) {
      const uint2 raw = *reinterpret_cast<const uint2 *>(x + o);
      T e[4];
      memcpy(e, &raw, 8);
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = to_f32(e[j]);
      return;
    }
    int4 acc = *reinterpret_cast<const int4 *>(part + o);
    for (int c = 1; c < C; ++c) {
      const int4 q = *reinterpret_cast<const int4 *>(part + c * cstride + o);
      acc.x += q.x;
      acc.y += q.y;
      acc.z += q.z;
      acc.w += q.w;
    }
    const float sx = xs[m];
    const float4 sw = *reinterpret_cast<const float4 *>(ws + col);
    v[0] = round_to<T>(__fmul_rn(__fmul_rn(static_cast<float>(acc.x), sx), sw.x));
    v[1] = round_to<T>(__fmul_rn(__fmul_rn(static_cast<float>(acc.y), sx), sw.y));
    v[2] = round_to<T>(__fmul_rn(__fmul_rn(static_cast<float>(acc.z), sx), sw.z));
    v[3] = round_to<T>(__fmul_rn(__fmul_rn(static_cast<float>(acc.w), sx), sw.w));
  }
};
template <typename T>
inline RowSrc<T> row_src(const void *x, int ld) {
  return RowSrc<T>{static_cast<const T *>(x), nullptr, nullptr, nullptr, 0, 1, ld};
}
template <typename T>
inline RowSrc<T> row_src_split(const int32_t *part, int C, const float *xs, const float *ws,
                               int M, int ld) {
  return RowSrc<T>{nullptr, part, xs, ws, static_cast<size_t>(M) * ld, C, ld};
}

// Rows of the inter-stage codec's payload, D values each (S8B_CODEC_* scheme), as a row
// source: load4 decodes exactly as s8b_codec_decode does, output rounded to T. For the -had
// schemes the 32 lanes of a warp must call load4 together on the 128 consecutive values of
// one block (lane l: values 4l .. 4l + 3), for the inverse Hadamard. A separate type (not a
// mode of RowSrc) so that kernels on plain or split rows carry none of this code.
template <typename T>
struct CodecSrc {
  const void *pay;
  const float *psc;
  int scheme, ld;
  static constexpr bool kCodec = true;
  __device__ __forceinline__ void load4(int m, int col, float v[4]) const {
    const int D = ld;
    if (scheme == S8B_CODEC_FP16) {
      const uint2 raw = *reinterpret_cast<const uint2 *>(static_cast<const T *>(pay) +
                                                         static_cast<size_t>(m) * D + col);
      T e[4];
      memcpy(e, &raw, 8);
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = to_f32(e[j]);
      return;
    }
    if (scheme == S8B_CODEC_INT8 || scheme == S8B_CODEC_INT8_HAD) {
      const char4 c = *reinterpret_cast<const char4 *>(static_cast<const int8_t *>(pay) +
                                                       static_cast<size_t>(m) * D + col);
      const float sc = psc[m];
      v[0] = __fmul_rn(static_cast<float>(c.x), sc);
      v[1] = __fmul_rn(static_cast<float>(c.y), sc);
      v[2] = __fmul_rn(static_cast<float>(c.z), sc);
      v[3] = __fmul_rn(static_cast<float>(c.w), sc);
    } else {
      const uint16_t pk = *reinterpret_cast<const uint16_t *>(
          static_cast<const uint8_t *>(pay) + static_cast<size_t>(m) * (D / 2) + col / 2);
      const float sc = psc[static_cast<size_t>(m) * (D / 128) + col / 128];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        int c = (pk >> (4 * i)) & 0xF;
        if (scheme == S8B_CODEC_NF4) {
          v[i] = __fmul_rn(nf4_value(c), sc);
        } else {
          c = c >= 8 ? c - 16 : c;
          v[i] = __fmul_rn(static_cast<float>(c), sc);
        }
      }
    }
    if (scheme == S8B_CODEC_INT8_HAD || scheme == S8B_CODEC_INT4_HAD) {
      fwht128_warp(v);
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = __fmul_rn(v[i], kHadScale);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = round_to<T>(v[i]);
  }
};
template <typename T>
inline CodecSrc<T> row_src_codec(const void *payload, const float *scales, int scheme, int D) {
  return CodecSrc<T>{payload, scales, scheme, D};
}

// ----------------------------------------------------------------------- quantizer -----
// Symmetric round-to-nearest: inv = qmax/amax, code = clamp(rint(x*inv)), scale = amax/qmax.
struct QParams {
  float inv, scale;
};
__device__ __forceinline__ QParams qparams(float amax, float qmax) {
  QParams p;
  if (amax > 0.0f) {
    p.inv = __fdiv_rn(qmax, amax);
    p.scale = __fdiv_rn(amax, qmax);
  } else {
    p.inv = 0.0f;
    p.scale = 1.0f;
  }
  return p;
}
__device__ __forceinline__ int qcode(float x, float inv, int qmax) {
  int c = __float2int_rn(__fmul_rn(x, inv));
  return c > qmax ? qmax : (c < -qmax ? -qmax : c);
}

// RMSNorm factor r = 1 / sqrt(f32(ss / n) + eps), ss accumulated in float64.
__device__ __forceinline__ float rms_factor(double ss, int n, float eps) {
  const float ms = static_cast<float>(ss / static_cast<double>(n));
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
}

}  // namespace s8b

#define S8B_DISPATCH_DTYPE(dtype, T, ...)                 \
  do {                                                    \
    if ((dtype) == S8B_BF16) {                            \
      using T = __nv_bfloat16;                            \
      __VA_ARGS__;                                        \
    } else if ((dtype) == S8B_FP16) {                     \
      using T = __half;                                   \
      __VA_ARGS__;                                        \
    } else {                                              \
      return S8B_ERR_DTYPE;                               \
    }                                                     \
  } while (0)
