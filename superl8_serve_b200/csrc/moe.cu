// Sparse-MoE FFN of a Qwen3-MoE layer (the reference's SparseMoE.forward,
// superl8serve/models/moe.py:88-141), in three launches around two grouped W8A8 GEMMs:
//
//   s8b_moe_route        router logits -> softmax -> top-k -> renormalise (one CTA per token),
//                        then the assignments grouped by expert (one CTA);
//   s8b_moe_gemm_grouped expert e's weights [N, K] applied to its rows [off[e], off[e+1])
//                        (dp4a on a shared-memory weight tile: every weight byte is read from
//                        HBM once, and experts without rows are skipped) — used for gate_up
//                        (rows gathered from the token activations) and for down (rows in
//                        place);
//   s8b_moe_combine      per token, the bf16 weighted contributions added in ascending
//                        expert index, as the reference's per-expert index_add_ loop does.
//
// At decode sizes (a few tokens per expert) the expert weights stream from HBM once per
// step, so the GEMMs are laid out like the dense dp4a GEMV: a warp owns 4 output rows, its
// lanes split K into 16-byte vectors, integer sums finish in a shuffle reduction.
#include "common.cuh"

namespace s8b {
namespace {

constexpr int kRouteThreads = 256;
constexpr int kMaxExperts = 256;
constexpr int kMaxTopK = 16;
constexpr int kMaxGroupTokens = 4096;

// ---------------------------------------------------------------------------- router ----
// Logits: lane j of a warp accumulates in float64 the exact products y[k]*g[e,k] for
// k = 256*i + 8*j + u (i ascending, u = 0..7), an xor butterfly joins the lanes, one rounding
// to float32. Softmax (warp 0): lane j holds experts j + 32c; max; e = exp_s8b(l - m);
// lane-order float32 sum and butterfly; p = e / S. Top-k: k rounds of a warp arg-max
// (larger value first, then lower index). Weights: p / max(sum in rank order, 1e-9),
// times the scaling factor, rounded to the activation dtype.
template <typename T>
__global__ void __launch_bounds__(kRouteThreads)
    moe_route_kernel(const T *__restrict__ y, const float *__restrict__ gate, int H, int E, int k,
                     int norm, float scaling, int32_t *__restrict__ topi, T *__restrict__ topw) {
  griddep_launch();
  griddep_wait();
  extern __shared__ float sm[];
  float *ys = sm;             // [H]
  float *logits = sm + H;     // [E]
  const int t = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const T *yr = y + static_cast<size_t>(t) * H;
  for (int i = threadIdx.x; i < H; i += kRouteThreads) ys[i] = to_f32(yr[i]);
  __syncthreads();
  const int steps = (H + 255) / 256;
  constexpr int kSteps = 8;  // gate loads issued together before the fp64 chain consumes them
  for (int e = warp; e < E; e += kRouteThreads / 32) {
    const float *g = gate + static_cast<size_t>(e) * H;
    double acc = 0.0;
    for (int i0 = 0; i0 < steps; i0 += kSteps) {
      float4 g0[kSteps], g1[kSteps];
#pragma unroll
      for (int q = 0; q < kSteps; ++q) {
        const int base = 256 * (i0 + q) + 8 * lane;
        if (i0 + q < steps && base < H) {  // H % 8 == 0: a lane's 8 elements all in or out
          g0[q] = __ldg(reinterpret_cast<const float4 *>(g + base));
          g1[q] = __ldg(reinterpret_cast<const float4 *>(g + base + 4));
        }
      }
#pragma unroll
      for (int q = 0; q < kSteps; ++q) {
        const int base = 256 * (i0 + q) + 8 * lane;
        if (i0 + q < steps && base < H) {
          const float gv[8] = {g0[q].x, g0[q].y, g0[q].z, g0[q].w,
                               g1[q].x, g1[q].y, g1[q].z, g1[q].w};
#pragma unroll
          for (int u = 0; u < 8; ++u)
            acc = __dadd_rn(acc, __dmul_rn(static_cast<double>(ys[base + u]),
                                           static_cast<double>(gv[u])));
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc = __dadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
    if (lane == 0) logits[e] = __double2float_rn(acc);
  }
  __syncthreads();
  if (warp != 0) return;
  constexpr int kC = kMaxExperts / 32;
  const int nc = (E + 31) / 32;
  float v[kC];
  float m = -INFINITY;
#pragma unroll
  for (int c = 0; c < kC; ++c) {
    const int e = lane + 32 * c;
    v[c] = (c < nc && e < E) ? logits[e] : -INFINITY;
    m = fmaxf(m, v[c]);
  }
  m = warp_max(m);
  float s = 0.0f;
#pragma unroll
  for (int c = 0; c < kC; ++c) {
    const int e = lane + 32 * c;
    const bool ok = c < nc && e < E;
    v[c] = ok ? exp_s8b(__fsub_rn(v[c], m)) : 0.0f;
    if (c < nc) s = __fadd_rn(s, v[c]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
#pragma unroll
  for (int c = 0; c < kC; ++c) v[c] = __fdiv_rn(v[c], s);
  // top-k selection
  unsigned taken = 0;
  float selv = 0.0f;  // lane r keeps the r-th selected value and index
  int seli = 0;
  for (int r = 0; r < k; ++r) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int c = 0; c < kC; ++c) {
      const int e = lane + 32 * c;
      // NaN ranks as -inf, and -inf still beats "nothing chosen" (bi = INT_MAX): every round
      // picks a valid expert index, whatever the inputs hold
      const float val = v[c] != v[c] ? -INFINITY : v[c];
      if (c < nc && e < E && !((taken >> c) & 1u) && (val > bv || (val == bv && e < bi))) {
        bv = val;
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    if (lane == r) {
      selv = bv;
      seli = bi;
    }
  }
  float tot = 0.0f;
  for (int r = 0; r < k; ++r) tot = __fadd_rn(tot, __shfl_sync(0xffffffffu, selv, r));
  tot = fmaxf(tot, 1e-9f);
  if (lane < k) {
    float w = norm ? __fdiv_rn(selv, tot) : selv;
    w = __fmul_rn(w, scaling);
    topi[static_cast<size_t>(t) * k + lane] = seli;
    topw[static_cast<size_t>(t) * k + lane] = from_f32<T>(w);
  }
}

// Assignments a = t*k + j grouped by expert, tokens ascending inside a group, from per-expert
// token bitmaps: rank of (e, t) = tokens before t in e's bitmap.
__global__ void __launch_bounds__(1024)
    moe_group_kernel(const int32_t *__restrict__ topi, int T_, int k, int E,
                     int32_t *__restrict__ offsets, int32_t *__restrict__ order,
                     int32_t *__restrict__ row_tok, int32_t *__restrict__ rowpos) {
  griddep_launch();
  griddep_wait();
  extern __shared__ uint32_t bm[];  // [E][W] token bitmaps, then offsets [E+1]
  const int W = (T_ + 31) / 32;
  int *off = reinterpret_cast<int *>(bm + static_cast<size_t>(E) * W);
  const int A = T_ * k;
  for (int i = threadIdx.x; i < E * W; i += blockDim.x) bm[i] = 0u;
  __syncthreads();
  for (int a = threadIdx.x; a < A; a += blockDim.x) {
    const int e = topi[a], t = a / k;
    atomicOr(&bm[e * W + (t >> 5)], 1u << (t & 31));
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int c = 0;
    for (int w = 0; w < W; ++w) c += __popc(bm[e * W + w]);
    off[e + 1] = c;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    off[0] = 0;
    for (int e = 0; e < E; ++e) off[e + 1] += off[e];
  }
  __syncthreads();
  for (int e = threadIdx.x; e <= E; e += blockDim.x) offsets[e] = off[e];
  for (int a = threadIdx.x; a < A; a += blockDim.x) {
    const int e = topi[a], t = a / k;
    const uint32_t *row = bm + e * W;
    int rank = __popc(row[t >> 5] & ((1u << (t & 31)) - 1u));
    for (int w = 0; w < (t >> 5); ++w) rank += __popc(row[w]);
    const int pos = off[e] + rank;
    order[pos] = a;
    row_tok[pos] = t;
    rowpos[a] = pos;
  }
}

// ------------------------------------------------------------------- grouped GEMM ----
// One CTA = (expert e, 32 consecutive weight rows). The CTA's weight tile (32 x K int8,
// contiguous in HBM) lands in shared memory through 16-byte cp.async copies issued by all
// threads at once (64 KB in flight for K = 2048), so the weight stream is read from HBM once
// whatever the expert's row count. Each pass then gathers 8 of the expert's token rows into
// shared memory (rows padded by 16 bytes, so the 8 rows' vectors at one K offset sit in
// different banks). Warp w owns tile rows 4w..4w+3; its lanes split K into 16-byte vectors,
// each lane applies its 4 weight vectors to the 8 token vectors (32 int32 sums), and a
// transpose reduction (31 shuffles) leaves lane l with the finished sum of output (tile row
// 4w + l/8, token l%8), which it stores. Slots past the expert's last row repeat that row and
// are not stored.
constexpr int kGWarps = 8;
constexpr int kGRows = 4;                   // weight rows per warp
constexpr int kGTile = kGWarps * kGRows;    // weight rows per CTA
constexpr int kGTok = 8;                    // token rows per pass (kGRows * kGTok == 32)

__device__ __forceinline__ int dot16(const int4 a, const int4 b, int acc) {
  acc = __dp4a(a.x, b.x, acc);
  acc = __dp4a(a.y, b.y, acc);
  acc = __dp4a(a.z, b.z, acc);
  acc = __dp4a(a.w, b.w, acc);
  return acc;
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

// v[0..31] of every lane -> lane l returns the sum over the warp of v[l] (integer adds).
__device__ __forceinline__ int transpose_reduce32(int (&v)[32], int lane) {
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) {
    const bool upper = (lane & s) != 0;
#pragma unroll
    for (int i = 0; i < s; ++i) {
      const int send = upper ? v[i] : v[i + s];
      const int keep = upper ? v[i + s] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, s);
    }
  }
  return v[0];
}

template <typename T>
__global__ void __launch_bounds__(kGWarps * 32, 2)
    moe_gemm_grouped_kernel(const int8_t *__restrict__ xq, const float *__restrict__ xs,
                            const int32_t *__restrict__ row_index, const int8_t *__restrict__ w,
                            const float *__restrict__ ws, const int32_t *__restrict__ offsets,
                            T *__restrict__ y, int N, int K) {
  extern __shared__ __align__(16) int4 gsm[];  // weight tile [kGTile][kv], tokens [kGTok][kv+1]
  __shared__ float xs_s[kGTok];
  griddep_launch();
  griddep_wait();  // offsets (and the activations) come from the preceding kernels
  const int e = blockIdx.y;
  const int lo = offsets[e], hi = offsets[e + 1];
  const int n0 = blockIdx.x * kGTile;
  if (lo >= hi || n0 >= N) return;  // uniform over the CTA
  const int rows = min(kGTile, N - n0);
  const int kv = K >> 4;
  int4 *wt = gsm;
  int4 *xt = gsm + kGTile * kv;
  {
    const int4 *src = reinterpret_cast<const int4 *>(w + (static_cast<size_t>(e) * N + n0) * K);
    const int nvec = rows * kv;
    for (int i = threadIdx.x; i < nvec; i += blockDim.x) cp_async16(wt + i, src + i);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r0 = warp * kGRows;
  const int4 *xv = reinterpret_cast<const int4 *>(xq);
  const float *wse = ws + static_cast<size_t>(e) * N + n0;
  int4 *wrow[kGRows];
#pragma unroll
  for (int r = 0; r < kGRows; ++r) wrow[r] = wt + min(r0 + r, rows - 1) * kv;
  for (int c0 = lo; c0 < hi; c0 += kGTok) {
    if (c0 != lo) __syncthreads();  // every warp is done with the previous pass's tokens
    for (int i = threadIdx.x; i < kGTok * kv; i += blockDim.x) {
      const int t = i / kv, j = i - t * kv;
      const int p = min(c0 + t, hi - 1);
      const int src = row_index ? row_index[p] : p;
      cp_async16(xt + t * (kv + 1) + j, xv + static_cast<size_t>(src) * kv + j);
    }
    if (threadIdx.x < kGTok) {
      const int p = min(c0 + static_cast<int>(threadIdx.x), hi - 1);
      xs_s[threadIdx.x] = xs[row_index ? row_index[p] : p];
    }
    cp_async_wait_all();
    __syncthreads();
    int acc[kGRows * kGTok];
#pragma unroll
    for (int i = 0; i < kGRows * kGTok; ++i) acc[i] = 0;
    for (int kk = lane; kk < kv; kk += 32) {
      int4 wr[kGRows];
#pragma unroll
      for (int r = 0; r < kGRows; ++r) wr[r] = wrow[r][kk];
#pragma unroll
      for (int t = 0; t < kGTok; ++t) {
        const int4 xr = xt[t * (kv + 1) + kk];
#pragma unroll
        for (int r = 0; r < kGRows; ++r) acc[r * kGTok + t] = dot16(wr[r], xr, acc[r * kGTok + t]);
      }
    }
    const int sum = transpose_reduce32(acc, lane);
    const int r = lane / kGTok, t = lane % kGTok;
    const int p = c0 + t, n = r0 + r;
    if (p < hi && n < rows) {
      const float v = __fmul_rn(__fmul_rn(static_cast<float>(sum), xs_s[t]), wse[n]);
      y[static_cast<size_t>(p) * N + n0 + n] = from_f32<T>(v);
    }
  }
}

// ------------------------------------------------------------------------ combine ----
template <typename T>
__global__ void __launch_bounds__(256)
    moe_combine_kernel(const T *__restrict__ contrib, const T *__restrict__ topw,
                       const int32_t *__restrict__ topi, const int32_t *__restrict__ rowpos,
                       T *__restrict__ out, int k, int H) {
  griddep_launch();
  griddep_wait();
  __shared__ int pos_s[kMaxTopK];
  __shared__ float w_s[kMaxTopK];
  const int t = blockIdx.x;
  if (threadIdx.x == 0) {
    // the token's k experts are distinct: order them by expert index (insertion sort)
    int ord[kMaxTopK];
    for (int j = 0; j < k; ++j) {
      int i = j;
      const int ej = topi[static_cast<size_t>(t) * k + j];
      while (i > 0 && topi[static_cast<size_t>(t) * k + ord[i - 1]] > ej) {
        ord[i] = ord[i - 1];
        --i;
      }
      ord[i] = j;
    }
    for (int r = 0; r < k; ++r) {
      const size_t a = static_cast<size_t>(t) * k + ord[r];
      pos_s[r] = rowpos[a];
      w_s[r] = to_f32(topw[a]);
    }
  }
  __syncthreads();
  for (int col = 4 * threadIdx.x; col < H; col += 4 * blockDim.x) {
    // all k contribution loads first, then the ordered sums
    uint2 raw[kMaxTopK];
#pragma unroll
    for (int r = 0; r < kMaxTopK; ++r)
      if (r < k)
        raw[r] = *reinterpret_cast<const uint2 *>(contrib + static_cast<size_t>(pos_s[r]) * H + col);
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int r = 0; r < kMaxTopK; ++r) {
      if (r >= k) break;
      T c[4];
      memcpy(c, &raw[r], 8);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float v = round_to<T>(__fmul_rn(to_f32(c[j]), w_s[r]));
        acc[j] = round_to<T>(__fadd_rn(acc[j], v));
      }
    }
    T o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = from_f32<T>(acc[j]);
    uint2 packed;
    memcpy(&packed, o, 8);
    *reinterpret_cast<uint2 *>(out + static_cast<size_t>(t) * H + col) = packed;
  }
}

}  // namespace
}  // namespace s8b

using namespace s8b;

extern "C" int s8b_moe_route(const void *y, int dtype, const float *gate, int T_, int H, int E,
                             int top_k, int norm_topk_prob, float routed_scaling, int32_t *topi,
                             void *topw, int32_t *expert_offsets, int32_t *sorted_assign,
                             int32_t *sorted_token, int32_t *assign_pos, void *stream) {
  if (!y || !gate || !topi || !topw || !expert_offsets || !sorted_assign || !sorted_token ||
      !assign_pos)
    return S8B_ERR_ARG;
  if (T_ < 0 || H <= 0 || H % 8 != 0 || E <= 0 || E > kMaxExperts || top_k <= 0 ||
      top_k > kMaxTopK || top_k > E || T_ > kMaxGroupTokens)
    return S8B_ERR_SHAPE;
  if (!aligned(gate, 16)) return S8B_ERR_ALIGN;
  const size_t route_smem = sizeof(float) * (static_cast<size_t>(H) + E);
  const size_t group_smem =
      sizeof(uint32_t) * static_cast<size_t>(E) * ((T_ + 31) / 32) + sizeof(int) * (E + 1);
  if (route_smem > 200 * 1024 || group_smem > 200 * 1024) return S8B_ERR_SHAPE;
  const cudaStream_t st = (cudaStream_t)stream;
  if (T_ == 0) {
    // no tokens: every expert group is empty
    cudaError_t e = cudaMemsetAsync(expert_offsets, 0, sizeof(int32_t) * (E + 1), st);
    if (e != cudaSuccess) {
      record_cuda_error(e);
      return S8B_ERR_CUDA;
    }
    return S8B_OK;
  }
  S8B_DISPATCH_DTYPE(dtype, TT, {
    ensure_smem(reinterpret_cast<const void *>(moe_route_kernel<TT>), route_smem);
    cudaError_t e = launch_pdl(moe_route_kernel<TT>, dim3(T_), dim3(kRouteThreads), route_smem,
                               st, static_cast<const TT *>(y), gate, H, E, top_k,
                               norm_topk_prob, routed_scaling, topi, static_cast<TT *>(topw));
    if (e != cudaSuccess) {
      record_cuda_error(e);
      return S8B_ERR_CUDA;
    }
  });
  int rc = check_launch();
  if (rc) return rc;
  ensure_smem(reinterpret_cast<const void *>(moe_group_kernel), group_smem);
  cudaError_t e = launch_pdl(moe_group_kernel, dim3(1), dim3(1024), group_smem, st,
                             static_cast<const int32_t *>(topi), T_, top_k, E, expert_offsets,
                             sorted_assign, sorted_token, assign_pos);
  if (e != cudaSuccess) {
    record_cuda_error(e);
    return S8B_ERR_CUDA;
  }
  return check_launch();
}

extern "C" int s8b_moe_gemm_grouped(const int8_t *xq, const float *xs, const int32_t *row_index,
                                    const int8_t *w, const float *ws,
                                    const int32_t *expert_offsets, void *y, int A, int N, int K,
                                    int E, int dtype, void *stream) {
  if (!xq || !xs || !w || !ws || !expert_offsets || !y) return S8B_ERR_ARG;
  if (A < 0 || N <= 0 || K <= 0 || K % 16 != 0 || E <= 0 || E > 65535) return S8B_ERR_SHAPE;
  if (!aligned(xq, 16) || !aligned(w, 16)) return S8B_ERR_ALIGN;
  if (A == 0) return S8B_OK;
  const size_t smem = static_cast<size_t>(kGTile) * K + static_cast<size_t>(kGTok) * (K + 16);
  if (smem > 200 * 1024) return S8B_ERR_SHAPE;
  const dim3 grid((N + kGTile - 1) / kGTile, E);
  S8B_DISPATCH_DTYPE(dtype, TT, {
    ensure_smem(reinterpret_cast<const void *>(moe_gemm_grouped_kernel<TT>), smem);
    cudaError_t e = launch_pdl(moe_gemm_grouped_kernel<TT>, grid, dim3(kGWarps * 32), smem,
                               (cudaStream_t)stream, xq, xs, row_index, w, ws, expert_offsets,
                               static_cast<TT *>(y), N, K);
    if (e != cudaSuccess) {
      record_cuda_error(e);
      return S8B_ERR_CUDA;
    }
  });
  return check_launch();
}

extern "C" int s8b_moe_combine(const void *contrib, const void *topw, const int32_t *topi,
                               const int32_t *assign_pos, void *out, int T_, int top_k, int H,
                               int dtype, void *stream) {
  if (!contrib || !topw || !topi || !assign_pos || !out) return S8B_ERR_ARG;
  if (T_ < 0 || H <= 0 || H % 4 != 0 || top_k <= 0 || top_k > kMaxTopK) return S8B_ERR_SHAPE;
  if (!aligned(contrib, 8) || !aligned(out, 8)) return S8B_ERR_ALIGN;
  if (T_ == 0) return S8B_OK;
  S8B_DISPATCH_DTYPE(dtype, TT, {
    cudaError_t e = launch_pdl(moe_combine_kernel<TT>, dim3(T_), dim3(256), 0,
                               (cudaStream_t)stream, static_cast<const TT *>(contrib),
                               static_cast<const TT *>(topw), topi, assign_pos,
                               static_cast<TT *>(out), top_k, H);
    if (e != cudaSuccess) {
      record_cuda_error(e);
      return S8B_ERR_CUDA;
    }
  });
  return check_launch();
}
