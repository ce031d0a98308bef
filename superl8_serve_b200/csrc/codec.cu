// Inter-stage activation codec: [a | b] rows -> (optional block-128 Hadamard) -> per-row
// (int8) or per-128-group (int4, nf4) absmax scales -> packed codes, and the inverse.
//
// The encoder's stores go wherever `payload` / `scales` point; for a pipeline boundary that
// is the next stage's receive buffer on another GPU (peer pointer or IPC mapping), so the
// codes cross NVLink as plain 128-byte coalesced stores straight from registers.
#include "common.cuh"

namespace s8b {
namespace {

constexpr int kCodecThreads = 256;

// Values k .. k+3 (k % 4 == 0) of row `row` of [a | b]: a is dtype rows or a GEMM's split-K
// partials summed and dequantized on load (then Da % 4 == 0, checked on the host).
template <typename T>
__device__ __forceinline__ void load4_ab(const RowSrc<T> &a, const T *b, int Da, int Db, int row,
                                         int k, float v[4]) {
  if (k + 4 <= Da && (Da & 3) == 0) {
    a.load4(row, k, v);
    return;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int kk = k + i;
    v[i] = kk < Da ? to_f32(a.x[static_cast<size_t>(row) * Da + kk])
                   : to_f32(b[static_cast<size_t>(row) * Db + (kk - Da)]);
  }
}

template <typename T>
__device__ __forceinline__ void store_ab(T *a, T *b, int Da, int Db, int row, int k, float v) {
  if (k < Da)
    a[static_cast<size_t>(row) * Da + k] = from_f32<T>(v);
  else
    b[static_cast<size_t>(row) * Db + (k - Da)] = from_f32<T>(v);
}

template <typename T>
__global__ void __launch_bounds__(kCodecThreads)
    encode_kernel(RowSrc<T> a, const T *__restrict__ b, int Da, int Db, int scheme,
                  void *__restrict__ payload, float *__restrict__ scales) {
  extern __shared__ float z[];  // [D] binary32 (int8 schemes)
  __shared__ float red[32];
  const int row = blockIdx.x;
  const int D = Da + Db;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  if (scheme == S8B_CODEC_FP16) {
    T *out = static_cast<T *>(payload) + static_cast<size_t>(row) * D;
    for (int k4 = threadIdx.x; k4 < D / 4; k4 += blockDim.x) {
      float v[4];
      load4_ab(a, b, Da, Db, row, 4 * k4, v);
#pragma unroll
      for (int i = 0; i < 4; ++i) out[4 * k4 + i] = from_f32<T>(v[i]);
    }
    return;
  }
  const bool had = scheme == S8B_CODEC_INT8_HAD || scheme == S8B_CODEC_INT4_HAD;
  if (scheme == S8B_CODEC_INT8 || scheme == S8B_CODEC_INT8_HAD) {
    float amax = 0.0f;
    if (had) {
      for (int blk = warp; blk < D / 128; blk += nwarps) {
        float v[4];
        load4_ab(a, b, Da, Db, row, blk * 128 + 4 * lane, v);
        fwht128_warp(v);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          v[i] = __fmul_rn(v[i], kHadScale);
          z[blk * 128 + 4 * lane + i] = v[i];
          amax = fmaxf(amax, fabsf(v[i]));
        }
      }
    } else {
      for (int k4 = threadIdx.x; k4 < D / 4; k4 += blockDim.x) {
        float v[4];
        load4_ab(a, b, Da, Db, row, 4 * k4, v);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          z[4 * k4 + i] = v[i];
          amax = fmaxf(amax, fabsf(v[i]));
        }
      }
    }
    amax = block_max(amax, red);
    const QParams p = qparams(amax, 127.0f);
    int8_t *out = static_cast<int8_t *>(payload) + static_cast<size_t>(row) * D;
    for (int k4 = threadIdx.x; k4 < D / 4; k4 += blockDim.x) {
      char4 c;
      c.x = static_cast<signed char>(qcode(z[4 * k4 + 0], p.inv, 127));
      c.y = static_cast<signed char>(qcode(z[4 * k4 + 1], p.inv, 127));
      c.z = static_cast<signed char>(qcode(z[4 * k4 + 2], p.inv, 127));
      c.w = static_cast<signed char>(qcode(z[4 * k4 + 3], p.inv, 127));
      reinterpret_cast<char4 *>(out)[k4] = c;
    }
    if (threadIdx.x == 0) scales[row] = p.scale;
    return;
  }
  // int4 / int4-had / nf4: one warp per 128-group.
  const bool nf4 = scheme == S8B_CODEC_NF4;
  uint8_t *out = static_cast<uint8_t *>(payload) + static_cast<size_t>(row) * (D / 2);
  for (int blk = warp; blk < D / 128; blk += nwarps) {
    float v[4];
    load4_ab(a, b, Da, Db, row, blk * 128 + 4 * lane, v);
    if (had) {
      fwht128_warp(v);
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = __fmul_rn(v[i], kHadScale);
    }
    float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    amax = warp_max(amax);
    int c[4];
    float scale;
    if (nf4) {
      // scale = absmax; code = nearest codebook entry to x / absmax (an all-zero group
      // gives scale 0 and code 7, the entry 0.0).
      scale = amax;
#pragma unroll
      for (int i = 0; i < 4; ++i) c[i] = nf4_code(amax > 0.0f ? __fdiv_rn(v[i], amax) : 0.0f);
    } else {
      const QParams p = qparams(amax, 7.0f);
      scale = p.scale;
#pragma unroll
      for (int i = 0; i < 4; ++i) c[i] = qcode(v[i], p.inv, 7);
    }
    const uint16_t packed = static_cast<uint16_t>(((c[0] & 0xF) | ((c[1] & 0xF) << 4)) |
                                                  (((c[2] & 0xF) | ((c[3] & 0xF) << 4)) << 8));
    reinterpret_cast<uint16_t *>(out + blk * 64)[lane] = packed;
    if (lane == 0) scales[static_cast<size_t>(row) * (D / 128) + blk] = scale;
  }
}

template <typename T>
__global__ void __launch_bounds__(kCodecThreads)
    decode_kernel(const void *__restrict__ payload, const float *__restrict__ scales, int Da,
                  int Db, int scheme, T *__restrict__ oa, T *__restrict__ ob) {
  const int row = blockIdx.x;
  const int D = Da + Db;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  if (scheme == S8B_CODEC_FP16) {
    const T *in = static_cast<const T *>(payload) + static_cast<size_t>(row) * D;
    for (int k = threadIdx.x; k < D; k += blockDim.x) store_ab(oa, ob, Da, Db, row, k, to_f32(in[k]));
    return;
  }
  if (scheme == S8B_CODEC_INT8) {
    const int8_t *in = static_cast<const int8_t *>(payload) + static_cast<size_t>(row) * D;
    const float s = scales[row];
    for (int k = threadIdx.x; k < D; k += blockDim.x)
      store_ab(oa, ob, Da, Db, row, k, __fmul_rn(static_cast<float>(in[k]), s));
    return;
  }
  const bool int8 = scheme == S8B_CODEC_INT8_HAD;
  const bool had = scheme == S8B_CODEC_INT8_HAD || scheme == S8B_CODEC_INT4_HAD;
  for (int blk = warp; blk < D / 128; blk += nwarps) {
    float v[4];
    if (int8) {
      const char4 c = reinterpret_cast<const char4 *>(static_cast<const int8_t *>(payload) +
                                                      static_cast<size_t>(row) * D + blk * 128)[lane];
      const float s = scales[row];
      v[0] = __fmul_rn(static_cast<float>(c.x), s);
      v[1] = __fmul_rn(static_cast<float>(c.y), s);
      v[2] = __fmul_rn(static_cast<float>(c.z), s);
      v[3] = __fmul_rn(static_cast<float>(c.w), s);
    } else {
      const uint16_t pk = reinterpret_cast<const uint16_t *>(
          static_cast<const uint8_t *>(payload) + static_cast<size_t>(row) * (D / 2) + blk * 64)[lane];
      const float s = scales[static_cast<size_t>(row) * (D / 128) + blk];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        int c = (pk >> (4 * i)) & 0xF;
        if (scheme == S8B_CODEC_NF4) {
          v[i] = __fmul_rn(nf4_value(c), s);
        } else {
          c = c >= 8 ? c - 16 : c;
          v[i] = __fmul_rn(static_cast<float>(c), s);
        }
      }
    }
    if (had) {
      fwht128_warp(v);
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = __fmul_rn(v[i], kHadScale);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) store_ab(oa, ob, Da, Db, row, blk * 128 + 4 * lane + i, v[i]);
  }
}

int check_codec(int T_, int Da, int Db, int scheme) {
  if (T_ < 0 || Da <= 0 || Db < 0) return S8B_ERR_SHAPE;
  if (scheme < S8B_CODEC_FP16 || scheme > S8B_CODEC_NF4) return S8B_ERR_DTYPE;
  const int D = Da + Db;
  if (D % 4 != 0) return S8B_ERR_SHAPE;
  if (scheme >= S8B_CODEC_INT8_HAD && (Da % 128 != 0 || Db % 128 != 0)) return S8B_ERR_SHAPE;
  if (D > 49152) return S8B_ERR_SHAPE;
  return S8B_OK;
}

}  // namespace
}  // namespace s8b

using namespace s8b;

extern "C" size_t s8b_codec_payload_bytes(int T_, int D, int scheme, int dtype) {
  (void)dtype;
  const size_t n = static_cast<size_t>(T_) * D;
  if (scheme == S8B_CODEC_FP16) return n * 2;
  if (scheme == S8B_CODEC_INT8 || scheme == S8B_CODEC_INT8_HAD) return n;
  return n / 2;
}

extern "C" size_t s8b_codec_scale_count(int T_, int D, int scheme) {
  if (scheme == S8B_CODEC_FP16) return 0;
  if (scheme == S8B_CODEC_INT8 || scheme == S8B_CODEC_INT8_HAD) return static_cast<size_t>(T_);
  return static_cast<size_t>(T_) * (D / 128);
}

extern "C" int s8b_codec_encode(const void *a, const void *b, int T_, int Da, int Db, int scheme,
                                void *payload, float *scales, int dtype, void *stream) {
  const int e = check_codec(T_, Da, Db, scheme);
  if (e) return e;
  if (!a || (Db > 0 && !b) || !payload || (scheme != S8B_CODEC_FP16 && !scales)) return S8B_ERR_ARG;
  if (!aligned(payload, 4)) return S8B_ERR_ALIGN;
  if (T_ == 0) return S8B_OK;
  const size_t smem = (scheme == S8B_CODEC_INT8 || scheme == S8B_CODEC_INT8_HAD)
                          ? static_cast<size_t>(Da + Db) * sizeof(float) : 0;
  S8B_DISPATCH_DTYPE(dtype, T, {
    auto kern = encode_kernel<T>;
    ensure_smem(reinterpret_cast<const void *>(kern), smem);
    kern<<<T_, kCodecThreads, smem, (cudaStream_t)stream>>>(
        row_src<T>(a, Da), static_cast<const T *>(b), Da, Db, scheme, payload, scales);
  });
  return check_launch();
}

extern "C" int s8b_codec_encode_split(const int32_t *part, int C, const float *xs,
                                      const float *ws, const void *b, int T_, int Da, int Db,
                                      int scheme, void *payload, float *scales, int dtype,
                                      void *stream) {
  const int e = check_codec(T_, Da, Db, scheme);
  if (e) return e;
  if (!part || !xs || !ws || (Db > 0 && !b) || !payload || (scheme != S8B_CODEC_FP16 && !scales))
    return S8B_ERR_ARG;
  if (C < 1 || C > 8 || Da % 4 != 0) return S8B_ERR_SHAPE;
  if (!aligned(payload, 4) || !aligned(part, 16) || !aligned(ws, 16)) return S8B_ERR_ALIGN;
  if (T_ == 0) return S8B_OK;
  const size_t smem = (scheme == S8B_CODEC_INT8 || scheme == S8B_CODEC_INT8_HAD)
                          ? static_cast<size_t>(Da + Db) * sizeof(float) : 0;
  S8B_DISPATCH_DTYPE(dtype, T, {
    auto kern = encode_kernel<T>;
    ensure_smem(reinterpret_cast<const void *>(kern), smem);
    kern<<<T_, kCodecThreads, smem, (cudaStream_t)stream>>>(
        row_src_split<T>(part, C, xs, ws, T_, Da), static_cast<const T *>(b), Da, Db, scheme,
        payload, scales);
  });
  return check_launch();
}

extern "C" int s8b_codec_decode(const void *payload, const float *scales, int T_, int Da, int Db,
                                int scheme, void *out_a, void *out_b, int dtype, void *stream) {
  const int e = check_codec(T_, Da, Db, scheme);
  if (e) return e;
  if (!payload || !out_a || (Db > 0 && !out_b) || (scheme != S8B_CODEC_FP16 && !scales))
    return S8B_ERR_ARG;
  if (!aligned(payload, 4)) return S8B_ERR_ALIGN;
  if (T_ == 0) return S8B_OK;
  S8B_DISPATCH_DTYPE(dtype, T,
                     decode_kernel<T><<<T_, kCodecThreads, 0, (cudaStream_t)stream>>>(
                         payload, scales, Da, Db, scheme, static_cast<T *>(out_a),
                         static_cast<T *>(out_b)));
  return check_launch();
}
