// Token sampler for the last stage (the reference's Sampler.forward,
// superl8serve/layers/sampler.py:22-86): repetition penalty, greedy or temperature, top-k,
// top-p, one draw. One CTA (1024 threads) per row; the row's scores live in a caller
// workspace (fp32, V per row) between passes.
//
// Every step is exact or a fixed binary32 operation, so the CPU oracle reproduces it:
//   x = f32(logits); each distinct id of history[0..pos] (pos = the row's input position,
//     history[pos] = the row's input id, written here first): x < 0 ? x * pen : x / pen;
//   greedy = argmax x (lowest index on ties); temperature 0 -> greedy;
//   s = x / max(temperature, 1e-5);
//   top-k (0 < k < V): keep s >= the k-th largest s (with multiplicity), the rest -inf;
//   e = exp_s8b(s - max s) (0 where s = -inf); q = floor(e * 2^32) as an integer mass;
//   top-p (p < 1): Q = sum q; keep e >= v*, v* the smallest e whose strictly larger
//     masses sum to <= floor(p * Q) (float64 product), the rest q = 0;
//   draw: u24 = splitmix64(seed + pos) >> 40; target = min(floor(u24 * Q' * 2^-24), Q' - 1)
//     in float64; the token is the first index whose running sum of q exceeds target.
// The k-th largest and v* are found by radix selection on order-preserving 32-bit keys
// (8 bits a pass), masses summed as 64-bit integers: no floating-point sum order anywhere.
#include "common.cuh"

namespace s8b {
namespace {

constexpr int kST = 1024;  // threads per row

__device__ __forceinline__ uint32_t order_key(float x) {
  const uint32_t b = __float_as_uint(x == 0.0f ? 0.0f : x);  // -0 and +0 compare equal
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ uint64_t mass_of(float e) {
  return static_cast<uint64_t>(static_cast<double>(e) * 4294967296.0);
}
__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
  uint64_t z = x + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__device__ uint64_t block_sum_u64(uint64_t v, uint64_t *red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  v = lane < (kST / 32) ? red[lane] : 0;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T>
__global__ void __launch_bounds__(kST)
    sample_kernel(const T *__restrict__ logits, int V, const float *__restrict__ temperature,
                  const int32_t *__restrict__ top_k, const float *__restrict__ top_p,
                  const float *__restrict__ penalty, const int32_t *__restrict__ input_ids,
                  const int32_t *__restrict__ positions, int32_t *__restrict__ history,
                  int history_cap, const uint64_t *__restrict__ seeds, float *__restrict__ ws,
                  int32_t *__restrict__ out) {
  extern __shared__ uint32_t seen[];  // V bits: ids already penalised
  __shared__ uint64_t red[32];
  __shared__ uint64_t mh[256];
  __shared__ uint32_t ch[256];
  __shared__ uint32_t sel_prefix;
  __shared__ uint64_t sel_above;
  __shared__ float fred[32];
  __shared__ int ired[32];
  griddep_launch();
  griddep_wait();
  const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const T *lr = logits + static_cast<size_t>(row) * V;
  float *x = ws + static_cast<size_t>(row) * V;
  const int pos = positions[row];
  const int in_id = input_ids[row];
  int32_t *hist = history + static_cast<size_t>(row) * history_cap;
  const int hl = min(pos + 1, history_cap);
  // x = f32(logits); history[pos] = the input id
  for (int i = tid; i < V; i += kST) x[i] = to_f32(lr[i]);
  for (int i = tid; i < (V + 31) / 32; i += kST) seen[i] = 0u;
  __syncthreads();
  if (tid == 0 && pos >= 0 && pos < history_cap) hist[pos] = in_id;
  __syncthreads();
  const float pen = penalty ? penalty[row] : 1.0f;
  if (pen != 1.0f) {
    for (int h = tid; h < hl; h += kST) {
      const int id = hist[h];
      if (id < 0 || id >= V) continue;
      const uint32_t bit = 1u << (id & 31);
      if (atomicOr(&seen[id >> 5], bit) & bit) continue;  // another position holds the same id
      const float v = x[id];
      x[id] = v < 0.0f ? __fmul_rn(v, pen) : __fdiv_rn(v, pen);
    }
  }
  __syncthreads();
  // greedy: max value, lowest index
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = tid; i < V; i += kST) {
    const float v = x[i];
    if (v > bv || (v == bv && i < bi)) {
      bv = v;
      bi = i;
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
  if (lane == 0) {
    fred[wid] = bv;
    ired[wid] = bi;
  }
  __syncthreads();
  if (wid == 0) {
    bv = fred[lane];
    bi = ired[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      fred[0] = bv;
      ired[0] = bi < V ? bi : 0;
    }
  }
  __syncthreads();
  const float temp = temperature[row];
  if (temp == 0.0f) {
    if (tid == 0) out[row] = ired[0];
    return;
  }
  const float tdiv = fmaxf(temp, 1e-5f);
  const float smax = __fdiv_rn(fred[0], tdiv);  // division is monotone: max of s
  for (int i = tid; i < V; i += kST) x[i] = __fdiv_rn(x[i], tdiv);
  __syncthreads();
  // top-k: the k-th largest key, by 8-bit radix passes
  const int k = top_k ? top_k[row] : 0;
  if (k > 0 && k < V) {
    uint32_t prefix = 0, mask = 0;
    int kk = k;
    for (int shift = 24; shift >= 0; shift -= 8) {
      if (tid < 256) ch[tid] = 0;
      __syncthreads();
      for (int i = tid; i < V; i += kST) {
        const uint32_t key = order_key(x[i]);
        if ((key & mask) == prefix) atomicAdd(&ch[(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (tid == 0) {
        int cum = 0, d = 255;
        for (; d > 0; --d) {
          if (cum + static_cast<int>(ch[d]) >= kk) break;
          cum += ch[d];
        }
        kk -= cum;
        sel_prefix = prefix | (static_cast<uint32_t>(d) << shift);
      }
      __syncthreads();
      prefix = sel_prefix;
      mask |= 255u << shift;
    }
    for (int i = tid; i < V; i += kST)
      if (order_key(x[i]) < prefix) x[i] = -INFINITY;
    __syncthreads();
  }
  // e = exp(s - max s) in place, integer masses
  uint64_t part = 0;
  for (int i = tid; i < V; i += kST) {
    const float s = x[i];
    const float e = s == -INFINITY ? 0.0f : exp_s8b(__fsub_rn(s, smax));
    x[i] = e;
    part += mass_of(e);
  }
  uint64_t Q = block_sum_u64(part, red);
  const float p = top_p ? top_p[row] : 1.0f;
  if (p < 1.0f) {
    const uint64_t Tp = static_cast<uint64_t>(floor(static_cast<double>(p) * static_cast<double>(Q)));
    uint32_t prefix = 0, mask = 0;
    uint64_t above = 0;  // mass of keys above the current prefix range
    for (int shift = 24; shift >= 0; shift -= 8) {
      if (tid < 256) {
        ch[tid] = 0;
        mh[tid] = 0;
      }
      __syncthreads();
      for (int i = tid; i < V; i += kST) {
        const float e = x[i];
        const uint32_t key = __float_as_uint(e);  // e >= 0: bits order like values
        if ((key & mask) == prefix) {
          const uint32_t d = (key >> shift) & 255u;
          atomicAdd(&ch[d], 1u);
          atomicAdd(reinterpret_cast<unsigned long long *>(&mh[d]),
                    static_cast<unsigned long long>(mass_of(e)));
        }
      }
      __syncthreads();
      if (tid == 0) {
        // the lowest non-empty digit whose largest key still has <= Tp of larger mass
        uint64_t run = above, best_above = above;
        int best = -1;
        for (int d = 255; d >= 0; --d) {
          if (ch[d] == 0) continue;
          if (run > Tp) break;
          best = d;
          best_above = run;
          run += mh[d];
        }
        if (best < 0) best = 0;  // cannot happen: the largest key always qualifies
        sel_prefix = prefix | (static_cast<uint32_t>(best) << shift);
        sel_above = best_above;
      }
      __syncthreads();
      prefix = sel_prefix;
      above = sel_above;
      mask |= 255u << shift;
    }
    part = 0;
    for (int i = tid; i < V; i += kST) {
      const float e = x[i];
      if (__float_as_uint(e) < prefix) x[i] = 0.0f;
      else part += mass_of(e);
    }
    Q = block_sum_u64(part, red);
  }
  // draw: inverse CDF in index order over contiguous per-thread segments. The greedy id is
  // stored first, so the row always has an output (Q is 0 only for NaN logits).
  if (tid == 0) out[row] = ired[0];
  if (Q == 0) return;
  __syncthreads();
  const uint64_t u24 = splitmix64(seeds[row] + static_cast<uint64_t>(static_cast<int64_t>(pos))) >> 40;
  uint64_t target = static_cast<uint64_t>(
      floor(static_cast<double>(u24) * static_cast<double>(Q) * 0x1p-24));
  if (target >= Q) target = Q - 1;
  const int seg = (V + kST - 1) / kST;
  const int lo = tid * seg, hi = min(V, lo + seg);
  uint64_t mine = 0;
  for (int i = lo; i < hi; ++i) mine += mass_of(x[i]);
  // exclusive scan of the segment masses
  uint64_t incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint64_t v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  __syncthreads();
  if (lane == 31) red[wid] = incl;
  __syncthreads();
  if (wid == 0) {
    uint64_t w = red[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint64_t v = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += v;
    }
    red[lane] = w;  // inclusive warp totals
  }
  __syncthreads();
  const uint64_t excl = (wid ? red[wid - 1] : 0) + incl - mine;
  if (mine > 0 && excl <= target && target < excl + mine) {
    uint64_t run = excl;
    for (int i = lo; i < hi; ++i) {
      run += mass_of(x[i]);
      if (run > target) {
        out[row] = i;
        break;
      }
    }
  }
}

}  // namespace
}  // namespace s8b

using namespace s8b;

extern "C" size_t s8b_sample_workspace_size(int M, int V) {
  return static_cast<size_t>(M > 0 ? M : 0) * (V > 0 ? V : 0) * sizeof(float);
}

extern "C" int s8b_sample(const void *logits, int dtype, int M, int V, const float *temperature,
                          const int32_t *top_k, const float *top_p, const float *penalty,
                          const int32_t *input_ids, const int32_t *positions, int32_t *history,
                          int history_cap, const uint64_t *seeds, void *workspace,
                          size_t workspace_bytes, int32_t *out, void *stream) {
  if (!logits || !temperature || !input_ids || !positions || !history || !seeds || !out)
    return S8B_ERR_ARG;
  if (M < 0 || V <= 0 || V > (1 << 24) || history_cap <= 0) return S8B_ERR_SHAPE;
  if (!workspace || workspace_bytes < s8b_sample_workspace_size(M, V)) return S8B_ERR_WORKSPACE;
  if (M == 0) return S8B_OK;
  const size_t smem = sizeof(uint32_t) * ((V + 31) / 32);
  if (smem > 160 * 1024) return S8B_ERR_SHAPE;
  S8B_DISPATCH_DTYPE(dtype, TT, {
    ensure_smem(reinterpret_cast<const void *>(sample_kernel<TT>), smem);
    cudaError_t e = launch_pdl(sample_kernel<TT>, dim3(M), dim3(kST), smem, (cudaStream_t)stream,
                               static_cast<const TT *>(logits), V, temperature, top_k, top_p,
                               penalty, input_ids, positions, history, history_cap, seeds,
                               static_cast<float *>(workspace), out);
    if (e != cudaSuccess) {
      record_cuda_error(e);
      return S8B_ERR_CUDA;
    }
  });
  return check_launch();
}
