// Attention side of the decode step on paged int8 KV.
//
// KV layout (one layer): codes [num_blocks, Hkv, bs, 128] int8, scales [num_blocks, Hkv, bs]
// fp32; token (block, off) of kv head g lives at row (block*Hkv + g)*bs + off, so the bs
// tokens of one (block, head) are 128*bs contiguous bytes. K is stored Hadamard-rotated; the
// query is rotated by the same orthonormal matrix, so q.k is unchanged.
//
// Decode attention runs in two kernels:
//  1. partitions: one CTA per (256-token partition, kv head, row). It stages the partition's
//     K and V codes with cp.async (144-byte K row pitch keeps 16-byte shared loads
//     conflict-free), forms exact int32 q.k dot products with dp4a, and accumulates
//     softmax numerator / denominator per query head in token order.
//  2. combine: one CTA per row merges the partitions in index order, writes the output in the
//     activation dtype and, fused, its per-token int8 codes for the o_proj GEMM.
// The fixed partition size and accumulation order make the result bit-identical to the CPU
// oracle (oracle/kernels.py: paged_decode).
#include <map>
#include <mutex>

#include "common.cuh"
#include "tcgen05.cuh"

namespace s8b {
namespace {

constexpr int kPart = 256;     // tokens per partition
constexpr int kKPitch = 144;   // shared-memory pitch of a K row (128 codes + 16 pad)
constexpr int kHd = 128;       // head dim handled by these kernels

__device__ __forceinline__ int slot_of(const int32_t *slot_mapping, const int32_t *block_table,
                                       int max_blocks, int bs, int m, int pos) {
  if (slot_mapping) return slot_mapping[m];
  return block_table[static_cast<size_t>(m) * max_blocks + pos / bs] * bs + pos % bs;
}

template <typename T>
__device__ __forceinline__ void load4(const T *p, float v[4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = to_f32(p[i]);
}

// Per-head RMSNorm over 128 elements held 4 per lane.
template <typename T>
__device__ __forceinline__ void head_rmsnorm(float v[4], const T *w, float eps) {
  double ss = 0.0;
#pragma unroll
  for (int i = 0; i < 4; ++i) ss += static_cast<double>(v[i]) * static_cast<double>(v[i]);
  ss = warp_sum_d(ss);
  const float r = rms_factor(ss, kHd, eps);
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    v[i] = round_to<T>(__fmul_rn(__fmul_rn(v[i], r), to_f32(w[4 * lane + i])));
}

// rotate-half RoPE: out[e] = x[e]*cos[e] + rot[e]*sin[e], rot = (-x[64:], x[:64]).
template <typename T>
__device__ __forceinline__ void head_rope(float v[4], const float *cs, const float *sn) {
  const int lane = threadIdx.x & 31;
  float o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = __shfl_xor_sync(0xffffffffu, v[i], 16);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int e = 4 * lane + i;
    const float rot = lane < 16 ? -o[i] : o[i];
    v[i] = round_to<T>(__fadd_rn(__fmul_rn(v[i], cs[e]), __fmul_rn(rot, sn[e])));
  }
}

// Quantize 128 values (4 per lane) to int8 with one scale; writes 4 codes per lane.
__device__ __forceinline__ float head_quant_store(const float v[4], int8_t *dst) {
  float a = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
  a = warp_max(a);
  const QParams p = qparams(a, 127.0f);
  char4 c;
  c.x = static_cast<signed char>(qcode(v[0], p.inv, 127));
  c.y = static_cast<signed char>(qcode(v[1], p.inv, 127));
  c.z = static_cast<signed char>(qcode(v[2], p.inv, 127));
  c.w = static_cast<signed char>(qcode(v[3], p.inv, 127));
  reinterpret_cast<char4 *>(dst)[threadIdx.x & 31] = c;
  return p.scale;
}

// K path shared by qkv_post and kv_write: Hadamard, round to T, quantize, store.
template <typename T>
__device__ __forceinline__ void store_k_row(float v[4], bool rotate, int8_t *kc, float *ks,
                                            size_t row) {
  if (rotate) {
    fwht128_warp(v);
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = round_to<T>(__fmul_rn(v[i], kHadScale));
  }
  const float sc = head_quant_store(v, kc + row * kHd);
  if ((threadIdx.x & 31) == 0) ks[row] = sc;
}

__device__ __forceinline__ void store_v_row(const float v[4], int8_t *vc, float *vs, size_t row) {
  const float sc = head_quant_store(v, vc + row * kHd);
  if ((threadIdx.x & 31) == 0) vs[row] = sc;
}

// --------------------------------------------------------------------------- qkv_post ----
// One warp per (token, head row): grid (ceil(HR / 8), M) x 256 threads.
constexpr int kQkvWarps = 8;
template <typename T>
__global__ void __launch_bounds__(kQkvWarps * 32)
    qkv_post_kernel(RowSrc<T> qkv, const int32_t *__restrict__ positions,
                    const float *__restrict__ cos_tab, const float *__restrict__ sin_tab,
                    const T *__restrict__ qn, const T *__restrict__ kn, float eps, int Hq,
                    int Hkv, int8_t *__restrict__ q_i8, float *__restrict__ q_s,
                    T *__restrict__ q_out, int8_t *__restrict__ kc, float *__restrict__ ks,
                    int8_t *__restrict__ vc, float *__restrict__ vs,
                    const int32_t *__restrict__ slot_mapping,
                    const int32_t *__restrict__ block_table, int max_blocks, int bs) {
  griddep_launch();  // the next kernel may start its prologue
  griddep_wait();    // launched with programmatic serialization
  const int m = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int HR = Hq + 2 * Hkv;
  const int hr = blockIdx.x * kQkvWarps + warp;
  if (hr >= HR) return;
  const int pos = positions[m];
  const int slot = slot_of(slot_mapping, block_table, max_blocks, bs, m, pos);
  const int blk = slot / bs, off = slot % bs;
  const float *cs = cos_tab + static_cast<size_t>(pos) * kHd;
  const float *sn = sin_tab + static_cast<size_t>(pos) * kHd;
  {
    float v[4];
    qkv.load4(m, hr * kHd + 4 * lane, v);
    if (hr < Hq) {
      head_rmsnorm<T>(v, qn, eps);
      head_rope<T>(v, cs, sn);
      if (q_out) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          q_out[(static_cast<size_t>(m) * Hq + hr) * kHd + 4 * lane + i] = from_f32<T>(v[i]);
      }
      fwht128_warp(v);
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = __fmul_rn(v[i], kHadScale);
      const float sc = head_quant_store(v, q_i8 + (static_cast<size_t>(m) * Hq + hr) * kHd);
      if (lane == 0) q_s[static_cast<size_t>(m) * Hq + hr] = sc;
    } else if (hr < Hq + Hkv) {
      const int g = hr - Hq;
      head_rmsnorm<T>(v, kn, eps);
      head_rope<T>(v, cs, sn);
      store_k_row<T>(v, true, kc, ks, (static_cast<size_t>(blk) * Hkv + g) * bs + off);
    } else {
      const int g = hr - Hq - Hkv;
      store_v_row(v, vc, vs, (static_cast<size_t>(blk) * Hkv + g) * bs + off);
    }
  }
}

// ----------------------------------------------------------------------- kv_write_paged ----
template <typename T>
__global__ void __launch_bounds__(256)
    kv_write_kernel(const T *__restrict__ k, const T *__restrict__ v, int8_t *__restrict__ kc,
                    float *__restrict__ ks, int8_t *__restrict__ vc, float *__restrict__ vs,
                    const int32_t *__restrict__ slot_mapping, int Hkv, int bs, int rotate_k) {
  const int t = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int slot = slot_mapping[t];
  const int blk = slot / bs, off = slot % bs;
  for (int hr = warp; hr < 2 * Hkv; hr += nwarps) {
    const int g = hr % Hkv;
    float x[4];
    const size_t row = (static_cast<size_t>(blk) * Hkv + g) * bs + off;
    if (hr < Hkv) {
      load4(k + (static_cast<size_t>(t) * Hkv + g) * kHd + 4 * lane, x);
      store_k_row<T>(x, rotate_k != 0, kc, ks, row);
    } else {
      load4(v + (static_cast<size_t>(t) * Hkv + g) * kHd + 4 * lane, x);
      store_v_row(x, vc, vs, row);
    }
  }
}

// ------------------------------------------------------------------ q rotate + quantize ----
template <typename T>
__global__ void __launch_bounds__(256) q_rotate_quant_kernel(const T *__restrict__ q, int Hq,
                                                             int8_t *__restrict__ q_i8,
                                                             float *__restrict__ q_s) {
  const int b = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  for (int h = warp; h < Hq; h += nwarps) {
    float v[4];
    const size_t base = (static_cast<size_t>(b) * Hq + h) * kHd;
    load4(q + base + 4 * lane, v);
    fwht128_warp(v);
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = __fmul_rn(v[i], kHadScale);
    const float sc = head_quant_store(v, q_i8 + base);
    if (lane == 0) q_s[static_cast<size_t>(b) * Hq + h] = sc;
  }
}

// ------------------------------------------------------------------- decode partitions ----
constexpr int kPartThreads = 512;
constexpr int kSlices = kPartThreads / 32;  // token slices of the P.V phase (one per warp)

template <int G>
struct PartSmem {
  // K and V codes [256 tokens][128], K with its 16-byte chunks XOR-swizzled by token % 8 so
  // that 8 lanes reading 8 consecutive tokens hit 8 different bank groups. After the scores and
  // the P.V loop, the same 64 KB hold the per-warp int32 partial sums [kSlices][G][128].
  static constexpr size_t kKV = 2 * kPart * kHd;
  static constexpr size_t kRed = static_cast<size_t>(kSlices) * G * kHd * 4;
  static constexpr size_t kRegion = kKV > kRed ? kKV : kRed;
  static constexpr size_t bytes = kRegion + 2 * kPart * 4 /*k,v scales*/ +
                                  static_cast<size_t>(G) * kPart * 4 /*e*/ +
                                  static_cast<size_t>(G) * kPart * 2 /*W*/ +
                                  static_cast<size_t>(G) * kHd /*q*/ +
                                  (4 * 8 + 64 + 8) * 4 /*per-head scalars, partial maxima*/ +
                                  kPart * 4 + 16 /*block row bases, flag*/;
};

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
template <typename T>
__device__ __forceinline__ float ldcg_act(const T *p) {
  const unsigned short bits = __ldcg(reinterpret_cast<const unsigned short *>(p));
  T v;
  memcpy(&v, &bits, sizeof(v));
  return to_f32(v);
}
__device__ __forceinline__ int dp2a_lo(int a, int b, int c) { return __dp2a_lo(a, b, c); }
__device__ __forceinline__ int dp2a_hi(int a, int b, int c) { return __dp2a_hi(a, b, c); }

// One CTA = one (256-token partition, kv head, row). Phases:
//  1. cp.async K (group 0) and V (group 1) of the partition's tokens; scales and q directly.
//  2. once K has landed: exact int32 q.k (dp4a), s = (f32(dot) * q_s*scale) * k_s; the V copy
//     is still in flight meanwhile.
//  3. per head: m = max s, e = exp(s - m), l = denominator in the fixed lane/butterfly order,
//     w = e * v_s, 15-bit weights W = rint(w * 32767/wmax).
//  4. once V has landed: o_int = sum W * v over this warp's 16 tokens for 4 channels x G heads
//     (dp2a: 2 tokens per instruction), partial sums reduced across the 16 warps in shared
//     memory (integer, exact), o = f32(o_int) * wmax/32767 -> workspace.
//  5. the CTA that finishes a (row, kv head) last (counter) merges its partitions in index
//     order into the output; the CTA that finishes a row last quantizes the row (o_proj input).
//     The host zeroes both counter arrays (one stream-ordered memset) before every launch of
//     these kernels, so a previous launch with another shape, or one that gave up, can never
//     leave a counter behind.
//
// Workspace layout: the status word sits at byte 0 for every shape, the counters follow at
// byte 256 (sized for this launch's B and Hq), the partials after them.
struct DecodeWs {
  int32_t *status;     // [1] S8B_ERR_TIMEOUT if a bounded wait of the tensor-core kernel gave up
  int32_t *cnt_group;  // [B*Hq] (row, kv head) completion counters (B*Hkv used)
  int32_t *cnt_row;    // [B]
  float *part_o;       // [B, Hq, P, 128]
  float *part_ml;      // [B, Hq, P, 2]
};

// Phase 5 shared by the partition kernels. The thread group that completes the last partition
// of its (row, kv head) merges the partitions in index order: M = max m_p, w_p = exp(m_p - M),
// L = sum w_p l_p, O = sum w_p o_p, out = dtype(O / L). The group that completes a row's last
// kv head quantizes the whole output row for the o_proj GEMM. Counters return to zero.
// Arrival follows the grid-barrier pattern: the group synchronises, then one thread fences
// (making the group's partial stores visible device-wide) and increments the counter; the
// last arriver fences again before the group reads the others' partials through L2.
// `tid` is the thread's index in the group of NTHR threads and `sync` synchronises exactly
// that group. `scratch` needs (G * P + G) floats, `red` 32 floats, `flag` one int.
struct CtaSync {
  __device__ __forceinline__ void operator()() const { __syncthreads(); }
};
template <int NTHR>
struct GroupSync {
  int id;
  __device__ __forceinline__ void operator()() const { tc::group_sync(id, NTHR); }
};

template <int NTHR, typename Sync>
__device__ __forceinline__ float group_max(float v, float *red, int tid, Sync sync) {
  v = warp_max(v);
  sync();
  if ((tid & 31) == 0) red[tid >> 5] = v;
  sync();
  v = (tid & 31) < NTHR / 32 ? red[tid & 31] : 0.0f;
  return warp_max(v);
}

template <typename T, int G, int NTHR, typename Sync>
__device__ __forceinline__ void merge_epilogue(float *scratch, float *red, int *flag,
                                               const DecodeWs &ws, int b, int g, int Hq, int Hkv,
                                               int P, int np, T *out, int8_t *out_q,
                                               float *out_s, int tid, Sync sync) {
  sync();
  if (tid == 0) {
    __threadfence();
    int32_t *c = ws.cnt_group + static_cast<size_t>(b) * Hkv + g;
    const int done = atomicAdd(c, 1) + 1;
    flag[0] = done == np;
    if (done == np) {
      *c = 0;
      __threadfence();
    }
  }
  sync();
  if (!flag[0]) return;
  // merge: per head h: M = max m_p, w_p = exp(m_p - M), L = sum w_p l_p, O = sum w_p o_p
  float *Wp = scratch;  // [G][P] merge weights
  float *Lh = Wp + G * P;
  if (tid < G) {
    const float *ml = ws.part_ml + (static_cast<size_t>(b) * Hq + g * G + tid) * P * 2;
    float M = -__int_as_float(0x7f800000);
    for (int q = 0; q < np; ++q) M = fmaxf(M, __ldcg(ml + 2 * q));
    float Ls = 0.0f;
    for (int q = 0; q < np; ++q) {
      const float w = exp_s8b(__fsub_rn(__ldcg(ml + 2 * q), M));
      Wp[tid * P + q] = w;
      Ls = __fadd_rn(Ls, __fmul_rn(w, __ldcg(ml + 2 * q + 1)));
    }
    Lh[tid] = Ls;
  }
  sync();
  for (int hd = tid; hd < G * kHd; hd += NTHR) {
    const int h = hd / kHd, d = hd % kHd;
    const float *po = ws.part_o + (static_cast<size_t>(b) * Hq + g * G + h) * P * kHd + d;
    float O = 0.0f;
    for (int q = 0; q < np; ++q) O = __fadd_rn(O, __fmul_rn(Wp[h * P + q], __ldcg(po + q * kHd)));
    out[static_cast<size_t>(b) * Hq * kHd + (g * G + h) * kHd + d] = from_f32<T>(__fdiv_rn(O, Lh[h]));
  }
  if (!out_q) return;
  sync();
  if (tid == 0) {
    __threadfence();
    const int done = atomicAdd(ws.cnt_row + b, 1) + 1;
    flag[0] = done == Hkv;
    if (done == Hkv) {
      ws.cnt_row[b] = 0;
      __threadfence();
    }
  }
  sync();
  if (!flag[0]) return;
  // quantize the whole output row (all heads) for the o_proj GEMM
  const T *row = out + static_cast<size_t>(b) * Hq * kHd;
  float amax = 0.0f;
  for (int i = tid; i < Hq * kHd; i += NTHR)  // written by other CTAs: read via L2
    amax = fmaxf(amax, fabsf(ldcg_act(row + i)));
  amax = group_max<NTHR>(amax, red, tid, sync);
  const QParams qp = qparams(amax, 127.0f);
  for (int i = tid; i < Hq * kHd; i += NTHR)
    out_q[static_cast<size_t>(b) * Hq * kHd + i] =
        static_cast<int8_t>(qcode(ldcg_act(row + i), qp.inv, 127));
  if (tid == 0) out_s[b] = qp.scale;
}

template <typename T, int G>
__global__ void __launch_bounds__(kPartThreads)
    attn_partition_kernel(const int8_t *__restrict__ q_i8, const float *__restrict__ q_s,
                          const int8_t *__restrict__ kc, const float *__restrict__ ks,
                          const int8_t *__restrict__ vc, const float *__restrict__ vs,
                          const int32_t *__restrict__ block_table,
                          const int32_t *__restrict__ context_lens, int Hq, int Hkv, int bs_log2,
                          int max_blocks, int P, float scale, DecodeWs ws, T *__restrict__ out,
                          int8_t *__restrict__ out_q, float *__restrict__ out_s) {
  using Sm = PartSmem<G>;
  const int p = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int n = context_lens[b];
  const int lo = p * kPart;
  if (lo >= n) return;
  const int cnt = min(kPart, n - lo);
  const int np = (n + kPart - 1) / kPart;
  const int bs = 1 << bs_log2;
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;

  extern __shared__ __align__(16) uint8_t smem[];
  int8_t *Ks = reinterpret_cast<int8_t *>(smem);
  int8_t *Vs = Ks + kPart * kHd;
  int32_t *Red = reinterpret_cast<int32_t *>(smem);  // reuses K/V after phase 4
  float *ksc = reinterpret_cast<float *>(smem + Sm::kRegion);
  float *vsc = ksc + kPart;
  float *E = vsc + kPart;                                   // [G][kPart]
  int16_t *W = reinterpret_cast<int16_t *>(E + G * kPart);  // [G][kPart]
  int8_t *Qs = reinterpret_cast<int8_t *>(W + G * kPart);   // [G][128]
  float *qsc = reinterpret_cast<float *>(Qs + G * kHd);     // [8]
  float *mx = qsc + 8;
  float *wsc = mx + 8;    // wmax / 32767
  float *lsum = wsc + 8;
  float *pmax = lsum + 8;   // [G][8] per-warp maxima of s, then of w
  float *winv = pmax + 64;  // [8] 32767 / wmax
  int *rowbase = reinterpret_cast<int *>(winv + 8);  // [kPart / bs] first row of each block
  int *flag = rowbase + kPart;

  // ---- phase 1: stage K then V (two cp.async groups) ----
  const int32_t *bt = block_table + static_cast<size_t>(b) * max_blocks + (lo >> bs_log2);
  const int nblk = (cnt + bs - 1) >> bs_log2;
  if (tid < nblk) rowbase[tid] = (bt[tid] * Hkv + g) << bs_log2;
  if (tid < G) qsc[tid] = __fmul_rn(q_s[static_cast<size_t>(b) * Hq + g * G + tid], scale);
  __syncthreads();
  for (int idx = tid; idx < cnt * 8; idx += kPartThreads) {
    const int t = idx >> 3, c = idx & 7;
    const size_t row = static_cast<size_t>(rowbase[t >> bs_log2] + (t & (bs - 1)));
    cp_async16(Ks + t * kHd + ((c ^ (t & 7)) * 16), kc + row * kHd + c * 16);
  }
  cp_async_commit();
  for (int idx = tid; idx < cnt * 8; idx += kPartThreads) {
    const int t = idx >> 3, c = idx & 7;
    const size_t row = static_cast<size_t>(rowbase[t >> bs_log2] + (t & (bs - 1)));
    cp_async16(Vs + t * kHd + c * 16, vc + row * kHd + c * 16);
  }
  cp_async_commit();
  if (tid < cnt) {
    const size_t row = static_cast<size_t>(rowbase[tid >> bs_log2] + (tid & (bs - 1)));
    ksc[tid] = ks[row];
    vsc[tid] = vs[row];
  }
  for (int idx = tid; idx < G * (kHd / 16); idx += kPartThreads) {
    const int h = idx / (kHd / 16), c = idx % (kHd / 16);
    reinterpret_cast<int4 *>(Qs + h * kHd)[c] =
        reinterpret_cast<const int4 *>(q_i8 + (static_cast<size_t>(b) * Hq + g * G + h) * kHd)[c];
  }
  cp_async_wait<1>();
  __syncthreads();

  // ---- phase 2: scores; each warp handles 32 consecutive tokens of one head ----
  for (int pr = tid; pr < G * kPart; pr += kPartThreads) {
    const int h = pr / kPart, t = pr % kPart;  // h is uniform within a warp
    float sv = -__int_as_float(0x7f800000);
    if (t < cnt) {
      const int8_t *kr = Ks + t * kHd;
      const int4 *qr = reinterpret_cast<const int4 *>(Qs + h * kHd);
      int acc = 0;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const int4 a = *reinterpret_cast<const int4 *>(kr + ((c ^ (t & 7)) * 16));
        const int4 q = qr[c];
        acc = __dp4a(a.x, q.x, acc);
        acc = __dp4a(a.y, q.y, acc);
        acc = __dp4a(a.z, q.z, acc);
        acc = __dp4a(a.w, q.w, acc);
      }
      sv = __fmul_rn(__fmul_rn(static_cast<float>(acc), qsc[h]), ksc[t]);
      E[pr] = sv;
    }
    const float wmx = warp_max(sv);
    if (lane == 0) pmax[h * 8 + (t >> 5)] = wmx;
  }
  __syncthreads();
  if (tid < G) {
    float m = pmax[tid * 8];
#pragma unroll
    for (int i = 1; i < 8; ++i) m = fmaxf(m, pmax[tid * 8 + i]);
    mx[tid] = m;
  }
  __syncthreads();
  // ---- phase 3: e = exp(s - m), value weights w = e * v_s, partial maxima of w ----
  for (int pr = tid; pr < G * kPart; pr += kPartThreads) {
    const int h = pr / kPart, t = pr % kPart;
    float w = 0.0f;
    if (t < cnt) {
      const float e = exp_s8b(__fsub_rn(E[pr], mx[h]));
      E[pr] = e;
      w = __fmul_rn(e, vsc[t]);
    } else {
      E[pr] = 0.0f;
    }
    const float wmx = warp_max(w);
    if (lane == 0) pmax[h * 8 + (t >> 5)] = wmx;
  }
  __syncthreads();
  if (tid < G) {
    float wm = pmax[tid * 8];
#pragma unroll
    for (int i = 1; i < 8; ++i) wm = fmaxf(wm, pmax[tid * 8 + i]);
    wsc[tid] = __fdiv_rn(wm, 32767.0f);
    winv[tid] = __fdiv_rn(32767.0f, wm);
  }
  __syncthreads();
  // ---- 15-bit weights (all threads); denominators (warp h, fixed lane/butterfly order) ----
  for (int pr = tid; pr < G * kPart; pr += kPartThreads) {
    const int h = pr / kPart, t = pr % kPart;
    int wq = 0;
    if (t < cnt) {
      wq = __float2int_rn(__fmul_rn(__fmul_rn(E[pr], vsc[t]), winv[h]));
      wq = wq < 0 ? 0 : (wq > 32767 ? 32767 : wq);
    }
    W[pr] = static_cast<int16_t>(wq);
  }
  if (warp < G) {
    const float *e = E + warp * kPart;
    float l = e[lane];
#pragma unroll
    for (int i = 1; i < kPart / 32; ++i) l = __fadd_rn(l, e[i * 32 + lane]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l = __fadd_rn(l, __shfl_xor_sync(0xffffffffu, l, o));
    if (lane == 0) lsum[warp] = l;
  }
  cp_async_wait<0>();
  __syncthreads();

  // ---- phase 4: o_int = sum_t W[h][t] * V[t][d], warp = 16-token slice, lane = 4 channels ----
  int acc[G][4];
#pragma unroll
  for (int h = 0; h < G; ++h)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[h][i] = 0;
  const int t_begin = warp * (kPart / kSlices);
  if (t_begin < cnt) {
#pragma unroll 2
    for (int t = t_begin; t < t_begin + kPart / kSlices; t += 2) {
      const int v0 = *reinterpret_cast<const int *>(Vs + t * kHd + 4 * lane);
      const int v1 = *reinterpret_cast<const int *>(Vs + (t + 1) * kHd + 4 * lane);
      const int lo01 = __byte_perm(v0, v1, 0x5140);  // (t,d) (t+1,d) (t,d+1) (t+1,d+1)
      const int hi23 = __byte_perm(v0, v1, 0x7362);  // same for d+2, d+3
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const int wpair = *reinterpret_cast<const int *>(W + h * kPart + t);
        acc[h][0] = dp2a_lo(wpair, lo01, acc[h][0]);
        acc[h][1] = dp2a_hi(wpair, lo01, acc[h][1]);
        acc[h][2] = dp2a_lo(wpair, hi23, acc[h][2]);
        acc[h][3] = dp2a_hi(wpair, hi23, acc[h][3]);
      }
    }
  }
  __syncthreads();  // all warps done with K/V: the region now holds the partial sums
#pragma unroll
  for (int h = 0; h < G; ++h)
    reinterpret_cast<int4 *>(Red + (static_cast<size_t>(warp) * G + h) * kHd)[lane] =
        make_int4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
  __syncthreads();
  for (int hd = tid; hd < G * kHd; hd += kPartThreads) {
    const int h = hd / kHd, d = hd % kHd;
    int o = 0;
#pragma unroll
    for (int sl = 0; sl < kSlices; ++sl) o += Red[(static_cast<size_t>(sl) * G + h) * kHd + d];
    const size_t hq = static_cast<size_t>(b) * Hq + g * G + h;
    ws.part_o[(hq * P + p) * kHd + d] = __fmul_rn(static_cast<float>(o), wsc[h]);
    if (d == 0) {
      ws.part_ml[(hq * P + p) * 2 + 0] = mx[h];
      ws.part_ml[(hq * P + p) * 2 + 1] = lsum[h];
    }
  }

  // ---- phase 5: the last partition of this (row, kv head) merges; the last group quantizes ----
  merge_epilogue<T, G, kPartThreads>(reinterpret_cast<float *>(smem), pmax, flag, ws, b, g, Hq,
                                     Hkv, P, np, out, out_q, out_s, tid, CtaSync{});
}

// ------------------------------------------------ tensor-core decode partitions ----
// Same partition arithmetic as attn_partition_kernel, with both contractions on tcgen05:
//  * q.k: D[token][head] (TMEM, int32) = K tile (A: 128 tokens x 128 ch, K-major, the SW128
//    image the cp.async staging writes) x Q (B: 16 rows = G heads + zero rows, K-major);
//    two 128-token tiles, 4 MMAs of K = 32 each;
//  * p.v: O^T[ch][head] = V^T (A: 128 channels x tokens, MN-major, the same swizzled rows) x
//    W (B: 16 rows x 256 tokens). The 15-bit weights are split into three signed byte planes,
//    W = 2^14*a + 2^7*b + c (a in {0,1}; b, c in 0..127), three MMA chains,
//    o = 2^14*D_a + 2^7*D_b + D_c: exact int32, hence bit-identical to the CUDA-core kernel
//    and the oracle.
// The per-token softmax work runs on 256 threads (thread = token, TMEM lane = token).
constexpr int kTcThreads = 256;
constexpr int kTcCols = 128;  // TMEM columns: S tile 0 | S tile 1 | O_a | O_b | O_c (16 each)

template <int G>
struct TcPartSmem {
  static constexpr int kK = 0;                     // K codes, later W planes (12 KB) + e
  static constexpr int kW = 0;                     // plane i at kW + 4096 i
  static constexpr int kE = 12288;                 // [G][256] floats (<= 8 KB)
  static constexpr int kV = kPart * kHd;           // V codes [256][128] (32 KB)
  static constexpr int kQ = kV + kPart * kHd;      // Q [16][128] (2 KB)
  static constexpr int kKsc = kQ + 16 * kHd;       // [256] floats
  static constexpr int kVsc = kKsc + kPart * 4;    // [256] floats
  static constexpr int kMisc = kVsc + kPart * 4;
  static constexpr int kMiscBytes = 1536;
  static constexpr size_t bytes = 1024 + kMisc + kMiscBytes;
};

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

template <typename T, int G>
__global__ void __launch_bounds__(kTcThreads)
    attn_partition_tc_kernel(const int8_t *__restrict__ q_i8, const float *__restrict__ q_s,
                             const int8_t *__restrict__ kc, const float *__restrict__ ks,
                             const int8_t *__restrict__ vc, const float *__restrict__ vs,
                             const int32_t *__restrict__ block_table,
                             const int32_t *__restrict__ context_lens, int Hq, int Hkv,
                             int bs_log2, int max_blocks, int P, float scale, DecodeWs ws,
                             T *__restrict__ out, int8_t *__restrict__ out_q,
                             float *__restrict__ out_s) {
  using L = TcPartSmem<G>;
  using namespace tc;
  const int p = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int n = context_lens[b];
  const int lo = p * kPart;
  if (lo >= n) return;
  const int cnt = min(kPart, n - lo);
  const int np = (n + kPart - 1) / kPart;
  const int bs = 1 << bs_log2;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  extern __shared__ uint8_t smem_raw[];
  uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  int8_t *Ks = reinterpret_cast<int8_t *>(sm + L::kK);
  int8_t *Vs = reinterpret_cast<int8_t *>(sm + L::kV);
  int8_t *Qs = reinterpret_cast<int8_t *>(sm + L::kQ);
  uint8_t *Wpl = sm + L::kW;
  float *E = reinterpret_cast<float *>(sm + L::kE);
  float *ksc = reinterpret_cast<float *>(sm + L::kKsc);
  float *vsc = reinterpret_cast<float *>(sm + L::kVsc);
  float *qsc = reinterpret_cast<float *>(sm + L::kMisc);  // [8]
  float *mx = qsc + 8, *wsc = mx + 8, *lsum = wsc + 8, *winv = lsum + 8;
  float *pmax = winv + 8;                                 // [G][8 warps]
  int *rowbase = reinterpret_cast<int *>(pmax + 64);      // [<= 256]
  int *flag = rowbase + 256;
  int *abort_flag = flag + 1;
  uint32_t *tmem_base = reinterpret_cast<uint32_t *>(flag + 2);
  uint64_t *bars = reinterpret_cast<uint64_t *>(flag + 4);  // [2], 8-byte aligned

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_base)), "r"(kTcCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // ---- phase 1: stage K, V (cp.async, swizzled), Q (swizzled, zero rows G..15), scales ----
  const int32_t *bt = block_table + static_cast<size_t>(b) * max_blocks + (lo >> bs_log2);
  const int nblk = (cnt + bs - 1) >> bs_log2;
  if (tid < nblk) rowbase[tid] = (bt[tid] * Hkv + g) << bs_log2;
  if (tid < G) qsc[tid] = __fmul_rn(q_s[static_cast<size_t>(b) * Hq + g * G + tid], scale);
  if (tid < 16 * 8) {
    const int h = tid >> 3, c = tid & 7;
    int4 v = make_int4(0, 0, 0, 0);
    if (h < G)
      v = reinterpret_cast<const int4 *>(q_i8 + (static_cast<size_t>(b) * Hq + g * G + h) * kHd)[c];
    *reinterpret_cast<int4 *>(Qs + h * kHd + ((c ^ (h & 7)) * 16)) = v;
  }
  __syncthreads();
  for (int idx = tid; idx < cnt * 8; idx += kTcThreads) {
    const int t = idx >> 3, c = idx & 7;
    const size_t row = static_cast<size_t>(rowbase[t >> bs_log2] + (t & (bs - 1)));
    cp_async16(Ks + t * kHd + ((c ^ (t & 7)) * 16), kc + row * kHd + c * 16);
  }
  cp_async_commit();
  for (int idx = tid; idx < cnt * 8; idx += kTcThreads) {
    const int t = idx >> 3, c = idx & 7;
    const size_t row = static_cast<size_t>(rowbase[t >> bs_log2] + (t & (bs - 1)));
    cp_async16(Vs + t * kHd + ((c ^ (t & 7)) * 16), vc + row * kHd + c * 16);
  }
  cp_async_commit();
  if (tid < cnt) {
    const size_t row = static_cast<size_t>(rowbase[tid >> bs_log2] + (tid & (bs - 1)));
    ksc[tid] = ks[row];
    vsc[tid] = vs[row];
  }
  cp_async_wait<1>();
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base;

  // ---- phase 2: S = K Q^T on the tensor cores ----
  if (tid == 0) {
    constexpr uint32_t id_s = i8_idesc(128, 16);
    const uint64_t qd = sw128_desc(smem_u32(Qs));
#pragma unroll
    for (int tile = 0; tile < 2; ++tile) {
      const uint64_t kd = sw128_desc(smem_u32(Ks + tile * 128 * kHd));
#pragma unroll
      for (int k = 0; k < 4; ++k) mma_i8(tmem + tile * 16, kd + 2 * k, qd + 2 * k, id_s, k > 0);
    }
    mma_commit(&bars[0]);
    mbar_wait(&bars[0], 0, abort_flag, ws.status);
  }
  __syncthreads();
  const bool ok1 = !*abort_flag;
  tc_fence_after();
  const int t = tid;  // token of this thread (= TMEM lane of its tile)
  float sv[G];
  if (ok1) {
    uint32_t v[16];
    tmem_ld16(tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16) + (warp >> 2) * 16, v);
    tmem_wait_ld();
#pragma unroll
    for (int h = 0; h < G; ++h)
      sv[h] = t < cnt ? __fmul_rn(__fmul_rn(static_cast<float>(static_cast<int32_t>(v[h])), qsc[h]), ksc[t])
                      : -__int_as_float(0x7f800000);
  }
  // ---- phase 3: softmax numerators, denominators, 15-bit value weights ----
#pragma unroll
  for (int h = 0; h < G; ++h) {
    const float m = warp_max(ok1 ? sv[h] : 0.0f);
    if (lane == 0) pmax[h * 8 + warp] = m;
  }
  __syncthreads();
  if (tid < G) {
    float m = pmax[tid * 8];
#pragma unroll
    for (int i = 1; i < 8; ++i) m = fmaxf(m, pmax[tid * 8 + i]);
    mx[tid] = m;
  }
  __syncthreads();
  float wv[G];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    float e = 0.0f;
    if (t < cnt) e = exp_s8b(__fsub_rn(sv[h], mx[h]));
    E[h * kPart + t] = e;
    wv[h] = t < cnt ? __fmul_rn(e, vsc[t]) : 0.0f;
    const float wm = warp_max(wv[h]);
    if (lane == 0) pmax[h * 8 + warp] = wm;
  }
  __syncthreads();
  if (tid < G) {
    float wm = pmax[tid * 8];
#pragma unroll
    for (int i = 1; i < 8; ++i) wm = fmaxf(wm, pmax[tid * 8 + i]);
    wsc[tid] = __fdiv_rn(wm, 32767.0f);
    winv[tid] = __fdiv_rn(32767.0f, wm);
  }
  __syncthreads();
  {  // W planes, K-major SW128 images of [16 rows][256 tokens] (two 128-token blocks each)
    const int blk = t >> 7, tt = t & 127;
#pragma unroll
    for (int h = 0; h < 16; ++h) {
      int wq = 0;
      if (h < G && t < cnt) {
        wq = __float2int_rn(__fmul_rn(wv[h < G ? h : 0], winv[h < G ? h : 0]));
        wq = wq < 0 ? 0 : (wq > 32767 ? 32767 : wq);
      }
      const int off = blk * 2048 + h * 128 + ((((tt >> 4) ^ (h & 7))) << 4) + (tt & 15);
      Wpl[off] = static_cast<uint8_t>(wq >> 14);
      Wpl[4096 + off] = static_cast<uint8_t>((wq >> 7) & 127);
      Wpl[8192 + off] = static_cast<uint8_t>(wq & 127);
    }
  }
  __syncthreads();
  if (warp < G) {
    const float *e = E + warp * kPart;
    float l = e[lane];
#pragma unroll
    for (int i = 1; i < kPart / 32; ++i) l = __fadd_rn(l, e[i * 32 + lane]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l = __fadd_rn(l, __shfl_xor_sync(0xffffffffu, l, o));
    if (lane == 0) lsum[warp] = l;
  }
  cp_async_wait<0>();
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // ---- phase 4: O^T = V^T W^T on the tensor cores (three byte planes of W) ----
  if (tid == 0 && ok1) {
    constexpr uint32_t id_pv = i8_idesc(128, 16, true, true, /*a_mn_major=*/true, false);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint64_t vd = sw128_desc(smem_u32(Vs + j * 32 * kHd));
#pragma unroll
      for (int pl = 0; pl < 3; ++pl) {
        const uint64_t wd = sw128_desc(smem_u32(Wpl + pl * 4096 + (j >> 2) * 2048)) + 2 * (j & 3);
        mma_i8(tmem + 32 + 16 * pl, vd, wd, id_pv, j > 0);
      }
    }
    mma_commit(&bars[1]);
    mbar_wait(&bars[1], 0, abort_flag, ws.status);
  }
  __syncthreads();
  const bool ok2 = !*abort_flag;
  tc_fence_after();
  if (ok2 && warp < 4) {
    uint32_t da[16], db[16], dc[16];
    const uint32_t lanes = static_cast<uint32_t>(warp * 32) << 16;
    tmem_ld16(tmem + lanes + 32, da);
    tmem_ld16(tmem + lanes + 48, db);
    tmem_ld16(tmem + lanes + 64, dc);
    tmem_wait_ld();
    const int d = warp * 32 + lane;
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const int o = static_cast<int32_t>(da[h]) * 16384 + static_cast<int32_t>(db[h]) * 128 +
                    static_cast<int32_t>(dc[h]);
      const size_t hq = static_cast<size_t>(b) * Hq + g * G + h;
      ws.part_o[(hq * P + p) * kHd + d] = __fmul_rn(static_cast<float>(o), wsc[h]);
    }
  }
  if (ok2 && tid < G) {
    const size_t hq = static_cast<size_t>(b) * Hq + g * G + tid;
    ws.part_ml[(hq * P + p) * 2 + 0] = mx[tid];
    ws.part_ml[(hq * P + p) * 2 + 1] = lsum[tid];
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTcCols) : "memory");
  if (!ok2) return;
  // ---- phase 5 ----
  merge_epilogue<T, G, kTcThreads>(reinterpret_cast<float *>(sm + L::kK), pmax, flag, ws, b, g,
                                   Hq, Hkv, P, np, out, out_q, out_s, tid, CtaSync{});
}

// ------------------------------------------ persistent warp-specialized decode ----
// One CTA per SM walks the work units (row b, kv head g, partition p) in a static round-robin.
// Roles:
//   warps 0, 14  producers (TMA issue from one warp tops out near 5.7 TB/s for 2 KB boxes):
//                per unit, warp 0 issues one 2-D TMA tensor copy per KV block of K plus one
//                for the G query rows, warp 14 one per KV block of V (the 128B swizzle lands
//                each row in the SW128 image the MMAs read) plus the K/V and query scales as
//                cp.async spread over its lanes, tracked by the same stage barrier; 3-stage
//                ring of 69 KB stages. Block-table rows (one per lane) are loaded three units
//                ahead.
//   warps 1, 15  MMA issuers (one thread each): warp 1 issues S = K Q^T as soon as a stage has
//                landed and an S buffer is free, warp 15 issues O^T = V^T W^T as soon as the
//                unit's weight planes are written and an O buffer is free. S and O are
//                double-buffered in TMEM (S: 2 x 32 columns, O: 2 x 48 columns).
//   warps 2-9    two softmax groups of 4 warps; group j takes the units with k % 2 == j, so
//                each group has two unit-times for its latency-bound chain (thread = TMEM
//                lane = tokens t and t + 128): scores, partition maxima, exp, the 15-bit
//                weights as three byte planes over the consumed K tile, the lane-order
//                denominators.
//   warps 10-13  epilogue: O planes -> per-partition partials in the workspace.
// No CTA waits for another: the partitions are merged afterwards by attn_merge_rows_kernel
// (a device-wide fence per unit here would stall the pipeline behind in-flight TMA traffic).
// The arithmetic per unit is exactly that of attn_partition_kernel. Every mbarrier wait is
// bounded; a timeout raises a CTA abort flag, which each role group turns into a uniform
// exit (barrier-reduce), and the workspace status word.
//
// p.v as one MMA of N = 48 per 32-token step: B rows 16*plane + head hold the byte planes of
// W = 2^14*a + 2^7*b + c, so D columns [0,16), [16,32), [32,48) are O_a, O_b, O_c.
namespace pk {
constexpr int kStages = 3;
constexpr int kStage = 70656;  // K/W/E 32 KB | V 32 KB | Q 2 KB | K, V scales 1 KB each | q scales
constexpr int kOffV = 32768, kOffQ = 65536, kOffKs = 67584, kOffVs = 68608, kOffQs = 69632;
constexpr int kOffMode = 70144;  // 1: the unit's blocks landed in reverse order (one 4-D copy)
constexpr int kWBlock = 6144;  // one 128-token block of the 48-row weight operand
constexpr int kOffE = 12288;   // e values [G][256] floats, after the two weight blocks
constexpr int kThreads = 512;
constexpr int kTmemCols = 256;
constexpr int kColO = 64;      // O buffer t at kColO + 48 t; S buffer t at 32 t
constexpr int kMisc = 2048;    // barriers, TMEM base, abort flag, stats, reductions
constexpr int kMaxRows = 1024; // context lengths cached in shared memory
constexpr size_t kSmem = 1024 + static_cast<size_t>(kStages) * kStage + kMisc + 4 * kMaxRows;
// multi-row launches also cache each row block's (first row | rows << 16) and longest context
constexpr size_t kSmemRows = kSmem + 8 * kMaxRows;
}  // namespace pk

// Walks units u = start, start + step, ... as (p, g, b) digits of u in radix (P, Hkv), with
// the step's digits computed once: advancing is adds and carries, no division (a per-unit
// division chain costs a single-warp role about a microsecond).
struct UnitIter {
  int p, g, b, dp, dg, db, P, Hkv;
  __device__ UnitIter(int start, int step, int P_, int Hkv_) : P(P_), Hkv(Hkv_) {
    p = start % P;
    g = (start / P) % Hkv;
    b = start / (P * Hkv);
    dp = step % P;
    dg = (step / P) % Hkv;
    db = step / (P * Hkv);
  }
  __device__ __forceinline__ void next() {
    p += dp;
    int c = p >= P;
    p -= c ? P : 0;
    g += dg + c;
    c = g >= Hkv;
    g -= c ? Hkv : 0;
    b += db + c;
  }
};

// EARLY: the kernel carries the early loads (run when `early` is set); without them it streams
// its steady state faster, which long unit lists need more than an early start.
template <typename T, int G, int R, bool EARLY>
__global__ void __launch_bounds__(pk::kThreads, 1)
    attn_persistent_kernel(const __grid_constant__ CUtensorMap map_k,
                           const __grid_constant__ CUtensorMap map_v,
                           const __grid_constant__ CUtensorMap map_q,
                           const __grid_constant__ CUtensorMap map_k4,
                           const __grid_constant__ CUtensorMap map_v4, int runs,
                           const float *__restrict__ q_s, const float *__restrict__ ks,
                           const float *__restrict__ vs, const int32_t *__restrict__ block_table,
                           const int32_t *__restrict__ context_lens, int B, int Hq, int Hkv,
                           int bs_log2, int max_blocks, int P, float scale, DecodeWs ws,
                           int early, const int8_t *__restrict__ q_i8,
                           const int32_t *__restrict__ row_blocks, int NB) {
  // R > 1 (prefill): a unit is (row block, kv head, partition); the block's rows are
  // consecutive rows of one sequence (one block-table row), and its R x G query heads are the
  // columns of the unit's S and O tiles (NC <= 16, the tiles' width), each column with its
  // own row's context. R = 1 (decode): a unit is (row, kv head, partition), NB = B.
  constexpr int NC = G * R;
  static_assert(NC <= 16, "a unit's query heads fill at most the 16 tile columns");
  static_assert(R == 1 || !EARLY, "early loads are for decode units");
  griddep_launch();  // the next kernel may start its prologue
  using namespace tc;
  using namespace pk;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *misc = sm + kStages * kStage;
  uint64_t *full = reinterpret_cast<uint64_t *>(misc);  // [3] stage loaded (tx bytes)
  uint64_t *empty = full + 3;                           // [3] stage free (p.v done + softmax done)
  uint64_t *wfull = full + 6;                           // [3] W planes of the stage written
  uint64_t *sfull = full + 9;                           // [2] S buffer holds a unit's scores
  uint64_t *sempty = full + 11;                         // [2] S buffer read (4 warp arrivals)
  uint64_t *ofull = full + 13;                          // [2] O buffer + stats ready
  uint64_t *oempty = full + 15;                         // [2] O buffer read (4 warp arrivals)
  uint64_t *drain = full + 17;                          // [2] MMA drains on exit (q.k, p.v)
  uint32_t *tmem_base = reinterpret_cast<uint32_t *>(misc + 256);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(misc + 260);
  float *stats = reinterpret_cast<float *>(misc + 512);  // [2][3][16]: m, l, wmax/32767
  float *red = reinterpret_cast<float *>(misc + 1024);   // [2 groups][2][4 warps][16 columns]
  int *ctx = reinterpret_cast<int *>(misc + kMisc);      // [B] context lengths
  int *rbi = ctx + kMaxRows;  // [NB] row block: first row | rows << 16 (R > 1)
  int *bmx = rbi + kMaxRows;  // [NB] row block's longest context (R > 1)
  // a unit's context (its longest row's), first row and row count
  auto unit_n = [&](int b) -> int {
    if constexpr (R == 1) return ctx[b];
    else return bmx[b];
  };
  auto unit_r0 = [&](int b) -> int {
    if constexpr (R == 1) return b;
    else return rbi[b] & 0xffff;
  };
  auto unit_nr = [&](int b) -> int {
    if constexpr (R == 1) return 1;
    else return rbi[b] >> 16;
  };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_base)), "r"(kTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < 3; ++i) {
      mbar_init(&full[i], 2 + 32);  // two expect_tx arrivals + one cp.async arrival per V lane
      mbar_init(&empty[i], 2);
      mbar_init(&wfull[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sfull[i], 1);
      mbar_init(&sempty[i], 4);
      mbar_init(&ofull[i], 2);
      mbar_init(&oempty[i], 4);
    }
    mbar_init(&drain[0], 1);
    mbar_init(&drain[1], 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  const int bs = 1 << bs_log2;
  const int nbu = kPart >> bs_log2;  // blocks of a full partition

  // ---------------------------------------------------------- producer helpers ----
  // This lane's KV block id for unit `it` of a row with context n (-1 past the end).
  auto block_id = [&](const UnitIter &it, int n) {
    if (it.b >= NB) return -1;
    const int nblk = (min(kPart, n - it.p * kPart) + bs - 1) >> bs_log2;
    if (lane >= nblk) return -1;
    return block_table[static_cast<size_t>(unit_r0(it.b)) * max_blocks +
                       ((it.p * kPart) >> bs_log2) + lane];
  };
  // Issues unit (p, g, b)'s K (warp 0, with the tx count of K and the query tile) or V and
  // the K/V scales (warp 14) into stage s; not the query tile, its scales or the V warp's
  // cp.async arrival. `blk` is this lane's block id, n the row's context length.
  auto issue_kv = [&](int p, int g, int b, int n, int blk, int s) {
    const bool vwarp = warp == 14;
    const int cnt = min(kPart, n - p * kPart);
    const int nblk = (cnt + bs - 1) >> bs_log2;
    const int row = (blk * Hkv + g) << bs_log2;  // this lane's block rows (lanes < nblk)
    // A full partition on consecutive block ids (ascending, or descending as the reference's
    // allocator hands them out) moves in one 4-D copy per tensor instead of nblk 2-D copies,
    // each of which costs its warp ~50 ns to issue. Descending runs land in reverse block
    // order; the softmax then stores its exponentials at the canonical token index.
    const int b0 = __shfl_sync(0xffffffffu, blk, 0);
    const bool asc = runs && nblk == nbu && __all_sync(0xffffffffu, lane >= nblk || blk == b0 + lane);
    // (reversed only for a partition with every token present: the softmax masks the
    // tokens past the context end by shared-memory row)
    const bool desc = runs && cnt == kPart && !asc &&
                      __all_sync(0xffffffffu, lane >= nblk || blk == b0 - lane);
    uint8_t *st = sm + s * kStage;
    if (lane == 0) {
      if (!vwarp) st[kOffMode] = desc ? 1 : 0;  // before the arrive that publishes the stage
      mbar_expect_tx(&full[s],
                     static_cast<uint32_t>(nblk * bs * kHd + (vwarp || R > 1 ? 0 : G * kHd)));
    }
    __syncwarp();
    if (asc || desc) {
      if (lane == 0)
        tma_load_4d(st + (vwarp ? kOffV : 0), vwarp ? &map_v4 : &map_k4, 0, 0, g,
                    desc ? b0 - (nbu - 1) : b0, &full[s]);
    } else if (lane < nblk) {
      tma_load_2d(st + (vwarp ? kOffV : 0) + lane * bs * kHd, vwarp ? &map_v : &map_k, 0, row,
                  &full[s]);
    }
    if (!vwarp) return;
    // scales: 16-byte chunks c of 4 tokens; chunk c of array a goes to lane c % 32
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = lane + 32 * (i & 1);  // chunk within the array
      const int j = (4 * c) >> bs_log2;   // smem block of that chunk
      const int rj = __shfl_sync(0xffffffffu, row, (desc ? nbu - 1 - j : j) & 31);
      if (4 * c < nblk * bs) {
        const float *src = (i < 2 ? ks : vs) + rj + ((4 * c) & (bs - 1));
        cp_async16(st + (i < 2 ? kOffKs : kOffVs) + 16 * c, src);
      }
    }
  };

  // Early phase (decode launches only): the kernel before this one writes each row's K/V at
  // position context_lens[b] - 1 and the queries, nothing else this kernel reads. The first
  // ring stages whose partitions end before that position are filled before waiting for it
  // (block tables, context lengths and older K/V are final before the step begins), so the
  // ring fills while that kernel still runs. Both producer warps walk the same units and stop
  // at the same one; `npre` stages then only need their query tile and scales.
  // Right after the wait the producers issue those stages' query tiles and scales (the first
  // q.k needs nothing else), and only then join the CTA barrier.
  int npre = 0;
  int pre_bg[kStages];  // (b * Hq + g * G) of the early stages: their query rows
  // query tile (warp 0) or query scales and the cp.async arrival (warp 14) of stage s, whose
  // query rows start at row qrow of the [B * Hq, 128] query array
  auto issue_q = [&](int qrow, int s) {
    uint8_t *st = sm + s * kStage;
    if (warp == 0) {
      if (lane == 0) tma_load_2d(st + kOffQ, &map_q, 0, qrow, &full[s]);
      return;
    }
    if (lane < G)
      asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(st + kOffQs + 4 * lane)),
                   "l"(q_s + static_cast<size_t>(qrow) + lane)
                   : "memory");
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(&full[s]))
                 : "memory");
  };
  // R > 1: the V warp copies the unit's query rows (column c = r * G + h at row c of the
  // 128B-swizzled tile, as a tensor copy would place it) and their scales with cp.async,
  // covered by its lanes' cp.async arrivals; the K warp has nothing to add.
  auto issue_q_rows = [&](int b, int g, int s) {
    if (warp == 0) return;
    uint8_t *st = sm + s * kStage;
    const int r0 = unit_r0(b), nr = unit_nr(b);
    for (int i = lane; i < NC * 8; i += 32) {
      const int c = i >> 3, ch = i & 7, r = c / G, h = c - (c / G) * G;
      if (r < nr)
        cp_async16(st + kOffQ + c * kHd + ((ch ^ (c & 7)) << 4),
                   q_i8 + (static_cast<size_t>(r0 + r) * Hq + g * G + h) * kHd + ch * 16);
    }
    if (lane < NC && lane / G < nr)
      asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(st + kOffQs + 4 * lane)),
                   "l"(q_s + static_cast<size_t>(r0 + lane / G) * Hq + g * G + lane % G)
                   : "memory");
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(&full[s]))
                 : "memory");
  };
  if (EARLY && R == 1 && early) {
    for (int i = threadIdx.x; i < B; i += kThreads) ctx[i] = __ldg(context_lens + i);
    __syncthreads();  // the context lengths are in and the stage barriers initialised
    if (warp == 0 || warp == 14) {
      UnitIter it(blockIdx.x, gridDim.x, P, Hkv);
      while (npre < kStages) {
        int n = it.b < B ? ctx[it.b] : 0;
        while (it.b < B && it.p * kPart >= n) {
          it.next();
          n = it.b < B ? ctx[it.b] : 0;
        }
        if (it.b >= B || (it.p + 1) * kPart >= n) break;  // holds the newest token
        issue_kv(it.p, it.g, it.b, n, block_id(it, n), npre);
        pre_bg[npre] = it.b * Hq + it.g * G;
        ++npre;
        it.next();
      }
    }
  }
  griddep_wait();  // launched with programmatic serialization: the prologue above overlaps
  if (EARLY && R == 1 && early && (warp == 0 || warp == 14)) {
#pragma unroll
    for (int j = 0; j < kStages; ++j)
      if (j < npre) issue_q(pre_bg[j], j);
  }
  if (!EARLY || R > 1 || !early)
    for (int i = threadIdx.x; i < B; i += kThreads) ctx[i] = context_lens[i];
  if constexpr (R > 1) {
    for (int i = threadIdx.x; i < NB; i += kThreads)
      rbi[i] = row_blocks[2 * i] | (min(row_blocks[2 * i + 1], R) << 16);
    __syncthreads();
    for (int i = threadIdx.x; i < NB; i += kThreads) {
      int m = 0;
      for (int r = 0; r < (rbi[i] >> 16); ++r) m = max(m, ctx[(rbi[i] & 0xffff) + r]);
      bmx[i] = m;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base;

  if (warp == 0 || warp == 14) {
    // ----------------------------------------------------------------- producers ----
    const bool vwarp = warp == 14;
    auto next_valid = [&](UnitIter &it) {
      while (it.b < NB && it.p * kPart >= unit_n(it.b)) it.next();
    };
    auto bid = [&](const UnitIter &it) { return block_id(it, it.b < NB ? unit_n(it.b) : 0); };
    // block-table rows three units ahead: under full HBM load a table miss takes a few us
    int k = 0;
    UnitIter i0(blockIdx.x, gridDim.x, P, Hkv);
    next_valid(i0);
    UnitIter i1 = i0;
    i1.next();
    next_valid(i1);
    UnitIter i2 = i1;
    i2.next();
    next_valid(i2);
    int blk0 = bid(i0), blk1 = bid(i1), blk2 = bid(i2);
    while (i0.b < NB) {
      const int blk = blk0;
      UnitIter i3 = i2;
      i3.next();
      next_valid(i3);
      blk0 = blk1;
      blk1 = blk2;
      blk2 = bid(i3);
      const int p = i0.p, g = i0.g, b = i0.b;
      const int s = k % kStages;
      bool ok = true;
      if (lane == 0 && k >= kStages)
        ok = mbar_wait(&empty[s], ((k / kStages) - 1) & 1, abort_flag, ws.status);
      if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
      if (k >= npre) {  // (early stages were issued whole before the CTA barrier)
        issue_kv(p, g, b, unit_n(b), blk, s);
        if constexpr (R == 1) issue_q(b * Hq + g * G, s);
        else issue_q_rows(b, g, s);
      }
      (void)vwarp;
      i0 = i1;
      i1 = i2;
      i2 = i3;
      ++k;
    }
    if (*abort_flag && lane == 0)  // let issued copies land before the CTA exits
      for (int j = k > kStages ? k - kStages : 0; j < k; ++j)
        mbar_drain(&full[j % kStages], (j / kStages) & 1);
  } else if (warp == 1) {
    // ------------------------------------------------------------- q.k MMA issuer ----
    if (lane == 0) {
      constexpr uint32_t id_s = i8_idesc(128, 16);
      int k = 0;
      for (UnitIter it(blockIdx.x, gridDim.x, P, Hkv); it.b < NB; it.next()) {
        if (it.p * kPart >= unit_n(it.b)) continue;
        const int s = k % kStages, t = k & 1;
        const bool ok = mbar_wait(&full[s], (k / kStages) & 1, abort_flag, ws.status) &&
                        (k < 2 || mbar_wait(&sempty[t], ((k >> 1) - 1) & 1, abort_flag, ws.status));
        if (!ok) break;
        tc_fence_after();
        uint8_t *st = sm + s * kStage;
        const uint64_t qd = sw128_desc(smem_u32(st + kOffQ));
#pragma unroll
        for (int tile = 0; tile < 2; ++tile) {
          const uint64_t kd = sw128_desc(smem_u32(st + tile * 128 * kHd));
#pragma unroll
          for (int i = 0; i < 4; ++i) mma_i8(tmem + 32 * t + 16 * tile, kd + 2 * i, qd + 2 * i, id_s, i > 0);
        }
        mma_commit(&sfull[t]);
        ++k;
      }
      mma_commit(&drain[0]);  // all MMAs issued by this thread have completed once this arrives
      mbar_drain(&drain[0], 0);
    }
  } else if (warp == 15) {
    // ------------------------------------------------------------- p.v MMA issuer ----
    // A thread of its own, so that q.k of later units never queues behind a p.v that waits
    // for its softmax.
    if (lane == 0) {
      constexpr uint32_t id_pv = i8_idesc(128, 48, true, true, /*a_mn_major=*/true, false);
      int k = 0;
      for (UnitIter it(blockIdx.x, gridDim.x, P, Hkv); it.b < NB; it.next()) {
        if (it.p * kPart >= unit_n(it.b)) continue;
        const int s = k % kStages, t = k & 1;
        const bool ok = mbar_wait(&wfull[s], (k / kStages) & 1, abort_flag, ws.status) &&
                        (k < 2 || mbar_wait(&oempty[t], ((k >> 1) - 1) & 1, abort_flag, ws.status));
        if (!ok) break;
        tc_fence_after();
        uint8_t *st = sm + s * kStage;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint64_t vd = sw128_desc(smem_u32(st + kOffV + i * 32 * kHd));
          const uint64_t wd = sw128_desc(smem_u32(st + (i >> 2) * kWBlock)) + 2 * (i & 3);
          mma_i8(tmem + kColO + 48 * t, vd, wd, id_pv, i > 0);
        }
        mma_commit(&ofull[t]);
        mma_commit(&empty[s]);
        ++k;
      }
      mma_commit(&drain[1]);
      mbar_drain(&drain[1], 0);
    }
  } else if (warp < 10) {
    // ------------------------------------------------------------------- softmax ----
    const int grp = (warp - 2) >> 2, q4 = warp & 3, tid = (threadIdx.x - 64) & 127;
    const int t0 = 32 * q4 + lane, t1 = t0 + 128;
    float *red_s = red + grp * 128, *red_w = red_s + 64;
    int k = 0;
    for (UnitIter it(blockIdx.x, gridDim.x, P, Hkv); it.b < NB; it.next()) {
      const int p = it.p, g = it.g, b = it.b;
      const int n = unit_n(b), lo = p * kPart;
      if (lo >= n) continue;
      if ((k & 1) != grp) {
        ++k;
        continue;
      }
      const int s = k % kStages, t = k & 1;
      bool ok = mbar_wait(&full[s], (k / kStages) & 1, abort_flag, ws.status) &&
                mbar_wait(&sfull[t], (k >> 1) & 1, abort_flag, ws.status) &&
                (k < 2 || mbar_wait(&oempty[t], ((k >> 1) - 1) & 1, abort_flag, ws.status));
      if (group_any(1 + grp, 128, !ok || *abort_flag)) break;
      // tokens of the partition inside each row's context (a row past the partition: 0)
      int cntr[R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if constexpr (R == 1) cntr[r] = min(kPart, n - lo);
        else cntr[r] = r < unit_nr(b) ? min(kPart, ctx[unit_r0(b) + r] - lo) : 0;
      }
      tc_fence_after();
      uint32_t a0[16], a1[16];
      tmem_ld16(tmem + (static_cast<uint32_t>(q4 * 32) << 16) + 32 * t, a0);
      tmem_ld16(tmem + (static_cast<uint32_t>(q4 * 32) << 16) + 32 * t + 16, a1);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sempty[t]);
      uint8_t *st = sm + s * kStage;
      const float *ksc = reinterpret_cast<const float *>(st + kOffKs);
      const float *vsc = reinterpret_cast<const float *>(st + kOffVs);
      const float *qsv = reinterpret_cast<const float *>(st + kOffQs);
      const float ks0 = ksc[t0], ks1 = ksc[t1], vs0 = vsc[t0], vs1 = vsc[t1];
      // canonical token index of shared-memory rows t0 and t1 (blocks reversed: see producers)
      const bool rev = st[kOffMode] != 0;
      const int nbu = kPart >> bs_log2;
      const int et0 = rev ? (((nbu - 1 - (t0 >> bs_log2)) << bs_log2) | (t0 & (bs - 1))) : t0;
      const int et1 = rev ? (((nbu - 1 - (t1 >> bs_log2)) << bs_log2) | (t1 & (bs - 1))) : t1;
      // column c (query head c % G of row c / G) masks by its row's context
      bool in0[NC], in1[NC];
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        in0[c] = et0 < cntr[c / G];
        in1[c] = et1 < cntr[c / G];
      }
      float s0[NC], s1[NC];
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        const float qsc = __fmul_rn(qsv[c], scale);
        s0[c] = in0[c] ? __fmul_rn(__fmul_rn(static_cast<float>(static_cast<int32_t>(a0[c])), qsc), ks0)
                       : -__int_as_float(0x7f800000);
        s1[c] = in1[c] ? __fmul_rn(__fmul_rn(static_cast<float>(static_cast<int32_t>(a1[c])), qsc), ks1)
                       : -__int_as_float(0x7f800000);
      }
      // The reductions below are latency chains on the stage's critical path: one redux per
      // column, all columns issued back to back.
      float red[NC];
#pragma unroll
      for (int c = 0; c < NC; ++c) red[c] = warp_max_redux(fmaxf(s0[c], s1[c]));
      if (lane == 0) {
#pragma unroll
        for (int c = 0; c < NC; ++c) red_s[q4 * 16 + c] = red[c];
      }
      group_sync(1 + grp, 128);
      // Loads, then arithmetic, then stores: a store into E may alias the reductions' shared
      // memory as far as the compiler knows, so interleaving them would chain the columns' exp
      // latencies one after another.
      float *E = reinterpret_cast<float *>(st + kOffE);
      float w0[NC], w1[NC], mh[NC];
#pragma unroll
      for (int c = 0; c < NC; ++c)
        mh[c] = fmaxf(fmaxf(red_s[c], red_s[16 + c]), fmaxf(red_s[32 + c], red_s[48 + c]));
      // All 2 NC exponentials unconditionally (a conditional call puts each ~400-cycle chain
      // behind its own branch; unconditional, they overlap). A masked token's score is -inf,
      // so its exp is 0 or NaN (a column with no token); the selects below drop it.
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        w0[c] = exp_s8b(__fsub_rn(s0[c], mh[c]));  // e, until stored
        w1[c] = exp_s8b(__fsub_rn(s1[c], mh[c]));
      }
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        w0[c] = in0[c] ? w0[c] : 0.0f;
        w1[c] = in1[c] ? w1[c] : 0.0f;
        E[c * kPart + et0] = w0[c];
        E[c * kPart + et1] = w1[c];
        w0[c] = in0[c] ? __fmul_rn(w0[c], vs0) : 0.0f;
        w1[c] = in1[c] ? __fmul_rn(w1[c], vs1) : 0.0f;
      }
#pragma unroll
      for (int c = 0; c < NC; ++c) red[c] = warp_max_redux(fmaxf(w0[c], w1[c]));
      if (lane == 0) {
#pragma unroll
        for (int c = 0; c < NC; ++c) red_w[q4 * 16 + c] = red[c];
      }
      group_sync(1 + grp, 128);
      float wm[NC];  // per-column weight maxima; their /32767 scales wait until after wfull
      int qa[NC], qb[NC];
#pragma unroll
      for (int c = 0; c < NC; ++c)
        wm[c] = fmaxf(fmaxf(red_w[c], red_w[16 + c]), fmaxf(red_w[32 + c], red_w[48 + c]));
      // 32767 / wm: one correctly rounded division per lane (lane c takes column c), shuffled
      // to the warp, instead of NC divisions in a row in every thread.
      float wl = 1.0f;
#pragma unroll
      for (int c = 0; c < NC; ++c) wl = lane == c ? wm[c] : wl;
      const float winv_l = __fdiv_rn(32767.0f, wl);
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        const float winv = __shfl_sync(0xffffffffu, winv_l, c);
        const int q0 = __float2int_rn(__fmul_rn(w0[c], winv));
        const int q1 = __float2int_rn(__fmul_rn(w1[c], winv));
        qa[c] = in0[c] ? (q0 < 0 ? 0 : (q0 > 32767 ? 32767 : q0)) : 0;
        qb[c] = in1[c] ? (q1 < 0 ? 0 : (q1 > 32767 ? 32767 : q1)) : 0;
      }
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        const int q0 = qa[c], q1 = qb[c];
        // rows 16*plane + c of the K-major SW128 weight operand; t0 lies in token block 0 and
        // t1 in block 1 at the same in-block position
        const int off = c * 128 + ((((t0 >> 4) ^ (c & 7))) << 4) + (t0 & 15);
        st[off] = static_cast<uint8_t>(q0 >> 14);
        st[2048 + off] = static_cast<uint8_t>((q0 >> 7) & 127);
        st[4096 + off] = static_cast<uint8_t>(q0 & 127);
        st[kWBlock + off] = static_cast<uint8_t>(q1 >> 14);
        st[kWBlock + 2048 + off] = static_cast<uint8_t>((q1 >> 7) & 127);
        st[kWBlock + 4096 + off] = static_cast<uint8_t>(q1 & 127);
      }
      fence_proxy_async_smem();
      group_sync(1 + grp, 128);
      if (tid == 0) mbar_arrive(&wfull[s]);
      float *st_t = stats + t * 48;
#pragma unroll
      for (int c = 0; c < NC; ++c) {  // denominators, lane order of the CUDA-core kernel
        if ((c & 3) != q4) continue;  // warp q4 takes columns q4, q4 + 4, ...
        const float *e = E + c * kPart;
        float l = e[lane];
#pragma unroll
        for (int i = 1; i < kPart / 32; ++i) l = __fadd_rn(l, e[i * 32 + lane]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l = __fadd_rn(l, __shfl_xor_sync(0xffffffffu, l, o));
        if (lane == 0) {
          st_t[c] = mh[c];
          st_t[16 + c] = l;
          st_t[32 + c] = __fdiv_rn(wm[c], 32767.0f);
        }
      }
      group_sync(1 + grp, 128);
      if (tid == 0) {
        mbar_arrive(&empty[s]);
        mbar_arrive(&ofull[t]);
      }
      ++k;
    }
  } else if (warp < 14) {
    // ------------------------------------------------------------------ epilogue ----
    const int q4 = warp & 3, tid = threadIdx.x - 320;
    const int d = 32 * q4 + lane;
    int k = 0;
    for (UnitIter it(blockIdx.x, gridDim.x, P, Hkv); it.b < NB; it.next()) {
      const int p = it.p, g = it.g, b = it.b;
      const int n = unit_n(b), lo = p * kPart;
      if (lo >= n) continue;
      const int t = k & 1;
      const bool ok = mbar_wait(&ofull[t], (k >> 1) & 1, abort_flag, ws.status);
      if (group_any(3, 128, !ok || *abort_flag)) break;
      tc_fence_after();
      uint32_t da[16], db[16], dc[16];
      const uint32_t lanes = static_cast<uint32_t>(q4 * 32) << 16;
      tmem_ld16(tmem + lanes + kColO + 48 * t, da);
      tmem_ld16(tmem + lanes + kColO + 48 * t + 16, db);
      tmem_ld16(tmem + lanes + kColO + 48 * t + 32, dc);
      tmem_wait_ld();
      const float *st_t = stats + t * 48;
      float wsc_c[NC];
#pragma unroll
      for (int c = 0; c < NC; ++c) wsc_c[c] = st_t[32 + c];
      float ml0 = 0.0f, ml1 = 0.0f;
      if (tid < NC) {
        ml0 = st_t[tid];
        ml1 = st_t[16 + tid];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&oempty[t]);
      const int r0 = unit_r0(b), nr = unit_nr(b);
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        const int r = c / G;
        if (R > 1 && (r >= nr || lo >= ctx[r0 + r])) continue;  // row past this partition
        const int o = static_cast<int32_t>(da[c]) * 16384 + static_cast<int32_t>(db[c]) * 128 +
                      static_cast<int32_t>(dc[c]);
        const size_t hq = static_cast<size_t>(r0 + r) * Hq + g * G + (c - r * G);
        ws.part_o[(hq * P + p) * kHd + d] = __fmul_rn(static_cast<float>(o), wsc_c[c]);
      }
      if (tid < NC) {
        const int r = tid / G;
        if (R == 1 || (r < nr && lo < ctx[r0 + r])) {
          const size_t hq = static_cast<size_t>(r0 + r) * Hq + g * G + (tid - r * G);
          ws.part_ml[(hq * P + p) * 2 + 0] = ml0;
          ws.part_ml[(hq * P + p) * 2 + 1] = ml1;
        }
      }
      ++k;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols) : "memory");
}

// The persistent kernel's decode form without the early loads and without multi-row units:
// the same roles, ring, tiles and arithmetic as attn_persistent_kernel<T, G, 1, false>, as a
// function of its own. Compiled apart from the early and multi-row code it streams its
// steady state faster for G <= 5 (measured 238.6 against 248.8 us per launch at 112 units
// per CTA, 27B at 16K context; 61.0 against 64.8 us for Qwen3-8B at batch 64), so those decode
// launches whose CTAs have many units take it. At G = 8 (Qwen3-30B-A3B) the template kernel
// is the faster one (142.8 against 165.7 us at batch 128, 4K context) and stays.
template <typename T, int G>
__global__ void __launch_bounds__(pk::kThreads, 1)
    attn_persistent_stream_kernel(const __grid_constant__ CUtensorMap map_k,
                           const __grid_constant__ CUtensorMap map_v,
                           const __grid_constant__ CUtensorMap map_q,
                           const __grid_constant__ CUtensorMap map_k4,
                           const __grid_constant__ CUtensorMap map_v4, int runs,
                           const float *__restrict__ q_s, const float *__restrict__ ks,
                           const float *__restrict__ vs, const int32_t *__restrict__ block_table,
                           const int32_t *__restrict__ context_lens, int B, int Hq, int Hkv,
                           int bs_log2, int max_blocks, int P, float scale, DecodeWs ws) {
  griddep_launch();  // the next kernel may start its prologue
  using namespace tc;
  using namespace pk;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *misc = sm + kStages * kStage;
  uint64_t *full = reinterpret_cast<uint64_t *>(misc);  // [3] stage loaded (tx bytes)
  uint64_t *empty = full + 3;                           // [3] stage free (p.v done + softmax done)
  uint64_t *wfull = full + 6;                           // [3] W planes of the stage written
  uint64_t *sfull = full + 9;                           // [2] S buffer holds a unit's scores
  uint64_t *sempty = full + 11;                         // [2] S buffer read (4 warp arrivals)
  uint64_t *ofull = full + 13;                          // [2] O buffer + stats ready
  uint64_t *oempty = full + 15;                         // [2] O buffer read (4 warp arrivals)
  uint64_t *drain = full + 17;                          // [2] MMA drains on exit (q.k, p.v)
  uint32_t *tmem_base = reinterpret_cast<uint32_t *>(misc + 256);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(misc + 260);
  float *stats = reinterpret_cast<float *>(misc + 512);  // [2][3][8]: m, l, wmax/32767
  float *red = reinterpret_cast<float *>(misc + 768);    // [2 groups][2][4 warps][8 heads]
  int *ctx = reinterpret_cast<int *>(misc + kMisc);      // [B] context lengths

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_base)), "r"(kTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < 3; ++i) {
      mbar_init(&full[i], 2 + 32);  // two expect_tx arrivals + one cp.async arrival per V lane
      mbar_init(&empty[i], 2);
      mbar_init(&wfull[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sfull[i], 1);
      mbar_init(&sempty[i], 4);
      mbar_init(&ofull[i], 2);
      mbar_init(&oempty[i], 4);
    }
    mbar_init(&drain[0], 1);
    mbar_init(&drain[1], 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  griddep_wait();  // launched with programmatic serialization: the prologue above overlaps
  for (int i = threadIdx.x; i < B; i += kThreads) ctx[i] = context_lens[i];
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base;
  const int bs = 1 << bs_log2;

  if (warp == 0 || warp == 14) {
    // ----------------------------------------------------------------- producers ----
    const bool vwarp = warp == 14;
    auto next_valid = [&](UnitIter &it) {
      while (it.b < B && it.p * kPart >= ctx[it.b]) it.next();
    };
    auto block_id = [&](const UnitIter &it) {  // this lane's KV block id (-1 past the end)
      if (it.b >= B) return -1;
      const int nblk = (min(kPart, ctx[it.b] - it.p * kPart) + bs - 1) >> bs_log2;
      if (lane >= nblk) return -1;
      return block_table[static_cast<size_t>(it.b) * max_blocks + ((it.p * kPart) >> bs_log2) +
                         lane];
    };
    const int nbu = kPart >> bs_log2;  // blocks of a full partition
    // block-table rows three units ahead: under full HBM load a table miss takes a few us
    int k = 0;
    UnitIter i0(blockIdx.x, gridDim.x, P, Hkv);
    next_valid(i0);
    UnitIter i1 = i0;
    i1.next();
    next_valid(i1);
    UnitIter i2 = i1;
    i2.next();
    next_valid(i2);
    int blk0 = block_id(i0), blk1 = block_id(i1), blk2 = block_id(i2);
    while (i0.b < B) {
      const int blk = blk0;
      UnitIter i3 = i2;
      i3.next();
      next_valid(i3);
      blk0 = blk1;
      blk1 = blk2;
      blk2 = block_id(i3);
      const int p = i0.p, g = i0.g, b = i0.b;
      const int cnt = min(kPart, ctx[b] - p * kPart);
      const int nblk = (cnt + bs - 1) >> bs_log2;
      const int row = (blk * Hkv + g) << bs_log2;  // this lane's block rows (lanes < nblk)
      // A full partition on consecutive block ids (ascending, or descending as the reference's
      // allocator hands them out) moves in one 4-D copy per tensor instead of nblk 2-D copies,
      // each of which costs its warp ~50 ns to issue. Descending runs land in reverse block
      // order; the softmax then stores its exponentials at the canonical token index.
      const int b0 = __shfl_sync(0xffffffffu, blk, 0);
      const bool asc = runs && nblk == nbu && __all_sync(0xffffffffu, lane >= nblk || blk == b0 + lane);
      // (reversed only for a partition with every token present: the softmax masks the
      // tokens past the context end by shared-memory row)
      const bool desc = runs && cnt == kPart && !asc &&
                        __all_sync(0xffffffffu, lane >= nblk || blk == b0 - lane);
      const int s = k % kStages;
      bool ok = true;
      if (lane == 0 && k >= kStages)
        ok = mbar_wait(&empty[s], ((k / kStages) - 1) & 1, abort_flag, ws.status);
      if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
      uint8_t *st = sm + s * kStage;
      if (lane == 0) {
        if (!vwarp) st[kOffMode] = desc ? 1 : 0;  // before the arrive that publishes the stage
        mbar_expect_tx(&full[s], static_cast<uint32_t>(nblk * bs * kHd + (vwarp ? 0 : G * kHd)));
      }
      __syncwarp();
      if (asc || desc) {
        if (lane == 0)
          tma_load_4d(st + (vwarp ? kOffV : 0), vwarp ? &map_v4 : &map_k4, 0, 0, g,
                      desc ? b0 - (nbu - 1) : b0, &full[s]);
      } else if (lane < nblk) {
        tma_load_2d(st + (vwarp ? kOffV : 0) + lane * bs * kHd, vwarp ? &map_v : &map_k, 0, row,
                    &full[s]);
      }
      if (!vwarp) {
        if (lane == 0) tma_load_2d(st + kOffQ, &map_q, 0, b * Hq + g * G, &full[s]);
        i0 = i1;
        i1 = i2;
        i2 = i3;
        ++k;
        continue;
      }
      // scales: 16-byte chunks c of 4 tokens; chunk c of array a goes to lane c % 32
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int c = lane + 32 * (i & 1);  // chunk within the array
        const int j = (4 * c) >> bs_log2;   // smem block of that chunk
        const int rj = __shfl_sync(0xffffffffu, row, (desc ? nbu - 1 - j : j) & 31);
        if (4 * c < nblk * bs) {
          const float *src = (i < 2 ? ks : vs) + rj + ((4 * c) & (bs - 1));
          cp_async16(st + (i < 2 ? kOffKs : kOffVs) + 16 * c, src);
        }
      }
      if (lane < G)  // the G query scales of this (row, kv head)
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(st + kOffQs + 4 * lane)),
                     "l"(q_s + static_cast<size_t>(b) * Hq + g * G + lane)
                     : "memory");
      asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(&full[s]))
                   : "memory");
      i0 = i1;
      i1 = i2;
      i2 = i3;
      ++k;
    }
    if (*abort_flag && lane == 0)  // let issued copies land before the CTA exits
      for (int j = k > kStages ? k - kStages : 0; j < k; ++j)
        mbar_drain(&full[j % kStages], (j / kStages) & 1);
  } else if (warp == 1) {
    // ------------------------------------------------------------- q.k MMA issuer ----
    if (lane == 0) {
      constexpr uint32_t id_s = i8_idesc(128, 16);
      int k = 0;
      for (UnitIter it(blockIdx.x, gridDim.x, P, Hkv); it.b < B; it.next()) {
        if (it.p * kPart >= ctx[it.b]) continue;
        const int s = k % kStages, t = k & 1;
        const bool ok = mbar_wait(&full[s], (k / kStages) & 1, abort_flag, ws.status) &&
                        (k < 2 || mbar_wait(&sempty[t], ((k >> 1) - 1) & 1, abort_flag, ws.status));
        if (!ok) break;
        tc_fence_after();
        uint8_t *st = sm + s * kStage;
        const uint64_t qd = sw128_desc(smem_u32(st + kOffQ));
#pragma unroll
        for (int tile = 0; tile < 2; ++tile) {
          const uint64_t kd = sw128_desc(smem_u32(st + tile * 128 * kHd));
#pragma unroll
          for (int i = 0; i < 4; ++i) mma_i8(tmem + 32 * t + 16 * tile, kd + 2 * i, qd + 2 * i, id_s, i > 0);
        }
        mma_commit(&sfull[t]);
        ++k;
      }
      mma_commit(&drain[0]);  // all MMAs issued by this thread have completed once this arrives
      mbar_drain(&drain[0], 0);
    }
  } else if (warp == 15) {
    // ------------------------------------------------------------- p.v MMA issuer ----
    // A thread of its own, so that q.k of later units never queues behind a p.v that waits
    // for its softmax.
    if (lane == 0) {
      constexpr uint32_t id_pv = i8_idesc(128, 48, true, true, /*a_mn_major=*/true, false);
      int k = 0;
      for (UnitIter it(blockIdx.x, gridDim.x, P, Hkv); it.b < B; it.next()) {
        if (it.p * kPart >= ctx[it.b]) continue;
        const int s = k % kStages, t = k & 1;
        const bool ok = mbar_wait(&wfull[s], (k / kStages) & 1, abort_flag, ws.status) &&
                        (k < 2 || mbar_wait(&oempty[t], ((k >> 1) - 1) & 1, abort_flag, ws.status));
        if (!ok) break;
        tc_fence_after();
        uint8_t *st = sm + s * kStage;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint64_t vd = sw128_desc(smem_u32(st + kOffV + i * 32 * kHd));
          const uint64_t wd = sw128_desc(smem_u32(st + (i >> 2) * kWBlock)) + 2 * (i & 3);
          mma_i8(tmem + kColO + 48 * t, vd, wd, id_pv, i > 0);
        }
        mma_commit(&ofull[t]);
        mma_commit(&empty[s]);
        ++k;
      }
      mma_commit(&drain[1]);
      mbar_drain(&drain[1], 0);
    }
  } else if (warp < 10) {
    // ------------------------------------------------------------------- softmax ----
    const int grp = (warp - 2) >> 2, q4 = warp & 3, tid = (threadIdx.x - 64) & 127;
    const int t0 = 32 * q4 + lane, t1 = t0 + 128;
    float *red_s = red + grp * 64, *red_w = red_s + 32;
    int k = 0;
    for (UnitIter it(blockIdx.x, gridDim.x, P, Hkv); it.b < B; it.next()) {
      const int p = it.p, g = it.g, b = it.b;
      const int n = ctx[b], lo = p * kPart;
      if (lo >= n) continue;
      if ((k & 1) != grp) {
        ++k;
        continue;
      }
      const int s = k % kStages, t = k & 1;
      bool ok = mbar_wait(&full[s], (k / kStages) & 1, abort_flag, ws.status) &&
                mbar_wait(&sfull[t], (k >> 1) & 1, abort_flag, ws.status) &&
                (k < 2 || mbar_wait(&oempty[t], ((k >> 1) - 1) & 1, abort_flag, ws.status));
      if (group_any(1 + grp, 128, !ok || *abort_flag)) break;
      const int cnt = min(kPart, n - lo);
      tc_fence_after();
      uint32_t a0[16], a1[16];
      tmem_ld16(tmem + (static_cast<uint32_t>(q4 * 32) << 16) + 32 * t, a0);
      tmem_ld16(tmem + (static_cast<uint32_t>(q4 * 32) << 16) + 32 * t + 16, a1);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sempty[t]);
      uint8_t *st = sm + s * kStage;
      const float *ksc = reinterpret_cast<const float *>(st + kOffKs);
      const float *vsc = reinterpret_cast<const float *>(st + kOffVs);
      const float *qsv = reinterpret_cast<const float *>(st + kOffQs);
      const float ks0 = ksc[t0], ks1 = ksc[t1], vs0 = vsc[t0], vs1 = vsc[t1];
      // canonical token index of shared-memory rows t0 and t1 (blocks reversed: see producers)
      const bool rev = st[kOffMode] != 0;
      const int nbu = kPart >> bs_log2;
      const int et0 = rev ? (((nbu - 1 - (t0 >> bs_log2)) << bs_log2) | (t0 & (bs - 1))) : t0;
      const int et1 = rev ? (((nbu - 1 - (t1 >> bs_log2)) << bs_log2) | (t1 & (bs - 1))) : t1;
      float s0[G], s1[G];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float qsc = __fmul_rn(qsv[h], scale);
        s0[h] = t0 < cnt ? __fmul_rn(__fmul_rn(static_cast<float>(static_cast<int32_t>(a0[h])), qsc), ks0)
                         : -__int_as_float(0x7f800000);
        s1[h] = t1 < cnt ? __fmul_rn(__fmul_rn(static_cast<float>(static_cast<int32_t>(a1[h])), qsc), ks1)
                         : -__int_as_float(0x7f800000);
      }
      // The reductions below are latency chains on the stage's critical path: one redux per
      // head, all heads issued back to back.
      float red[G];
#pragma unroll
      for (int h = 0; h < G; ++h) red[h] = warp_max_redux(fmaxf(s0[h], s1[h]));
      if (lane == 0) {
#pragma unroll
        for (int h = 0; h < G; ++h) red_s[q4 * 8 + h] = red[h];
      }
      group_sync(1 + grp, 128);
      // Loads, then arithmetic, then stores: a store into E may alias the reductions' shared
      // memory as far as the compiler knows, so interleaving them would chain the heads' exp
      // latencies one after another.
      float *E = reinterpret_cast<float *>(st + kOffE);
      float w0[G], w1[G], mh[G];
#pragma unroll
      for (int h = 0; h < G; ++h)
        mh[h] = fmaxf(fmaxf(red_s[h], red_s[8 + h]), fmaxf(red_s[16 + h], red_s[24 + h]));
      // All 2G exponentials unconditionally (a conditional call puts each ~400-cycle chain
      // behind its own branch; unconditional, they overlap). A masked token's score is -inf,
      // so its exp is 0 either way; the select below keeps the CUDA-core kernel's form.
#pragma unroll
      for (int h = 0; h < G; ++h) {
        w0[h] = exp_s8b(__fsub_rn(s0[h], mh[h]));  // e, until stored
        w1[h] = exp_s8b(__fsub_rn(s1[h], mh[h]));
      }
#pragma unroll
      for (int h = 0; h < G; ++h) {
        w0[h] = t0 < cnt ? w0[h] : 0.0f;
        w1[h] = t1 < cnt ? w1[h] : 0.0f;
        E[h * kPart + et0] = w0[h];
        E[h * kPart + et1] = w1[h];
        w0[h] = t0 < cnt ? __fmul_rn(w0[h], vs0) : 0.0f;
        w1[h] = t1 < cnt ? __fmul_rn(w1[h], vs1) : 0.0f;
      }
#pragma unroll
      for (int h = 0; h < G; ++h) red[h] = warp_max_redux(fmaxf(w0[h], w1[h]));
      if (lane == 0) {
#pragma unroll
        for (int h = 0; h < G; ++h) red_w[q4 * 8 + h] = red[h];
      }
      group_sync(1 + grp, 128);
      float wm[G];  // per-head weight maxima; their /32767 scales wait until after wfull
      int qa[G], qb[G];
#pragma unroll
      for (int h = 0; h < G; ++h)
        wm[h] = fmaxf(fmaxf(red_w[h], red_w[8 + h]), fmaxf(red_w[16 + h], red_w[24 + h]));
      // 32767 / wm: one correctly rounded division per lane (lane h takes head h), shuffled to
      // the warp, instead of G divisions in a row in every thread.
      float wl = 1.0f;
#pragma unroll
      for (int h = 0; h < G; ++h) wl = lane == h ? wm[h] : wl;
      const float winv_l = __fdiv_rn(32767.0f, wl);
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float winv = __shfl_sync(0xffffffffu, winv_l, h);
        const int q0 = __float2int_rn(__fmul_rn(w0[h], winv));
        const int q1 = __float2int_rn(__fmul_rn(w1[h], winv));
        qa[h] = t0 < cnt ? (q0 < 0 ? 0 : (q0 > 32767 ? 32767 : q0)) : 0;
        qb[h] = t1 < cnt ? (q1 < 0 ? 0 : (q1 > 32767 ? 32767 : q1)) : 0;
      }
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const int q0 = qa[h], q1 = qb[h];
        // rows 16*plane + h of the K-major SW128 weight operand; t0 lies in token block 0 and
        // t1 in block 1 at the same in-block position
        const int off = h * 128 + ((((t0 >> 4) ^ (h & 7))) << 4) + (t0 & 15);
        st[off] = static_cast<uint8_t>(q0 >> 14);
        st[2048 + off] = static_cast<uint8_t>((q0 >> 7) & 127);
        st[4096 + off] = static_cast<uint8_t>(q0 & 127);
        st[kWBlock + off] = static_cast<uint8_t>(q1 >> 14);
        st[kWBlock + 2048 + off] = static_cast<uint8_t>((q1 >> 7) & 127);
        st[kWBlock + 4096 + off] = static_cast<uint8_t>(q1 & 127);
      }
      fence_proxy_async_smem();
      group_sync(1 + grp, 128);
      if (tid == 0) mbar_arrive(&wfull[s]);
      float *st_t = stats + t * 24;
#pragma unroll
      for (int h = 0; h < G; ++h) {  // denominators, lane order of the CUDA-core kernel
        if ((h & 3) != q4) continue;  // warp q4 takes heads q4, q4 + 4
        const float *e = E + h * kPart;
        float l = e[lane];
#pragma unroll
        for (int i = 1; i < kPart / 32; ++i) l = __fadd_rn(l, e[i * 32 + lane]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l = __fadd_rn(l, __shfl_xor_sync(0xffffffffu, l, o));
        if (lane == 0) {
          st_t[h] = mh[h];
          st_t[8 + h] = l;
          st_t[16 + h] = __fdiv_rn(wm[h], 32767.0f);
        }
      }
      group_sync(1 + grp, 128);
      if (tid == 0) {
        mbar_arrive(&empty[s]);
        mbar_arrive(&ofull[t]);
      }
      ++k;
    }
  } else if (warp < 14) {
    // ------------------------------------------------------------------ epilogue ----
    const int q4 = warp & 3, tid = threadIdx.x - 320;
    const int d = 32 * q4 + lane;
    int k = 0;
    for (UnitIter it(blockIdx.x, gridDim.x, P, Hkv); it.b < B; it.next()) {
      const int p = it.p, g = it.g, b = it.b;
      const int n = ctx[b], lo = p * kPart;
      if (lo >= n) continue;
      const int t = k & 1;
      const bool ok = mbar_wait(&ofull[t], (k >> 1) & 1, abort_flag, ws.status);
      if (group_any(3, 128, !ok || *abort_flag)) break;
      tc_fence_after();
      uint32_t da[16], db[16], dc[16];
      const uint32_t lanes = static_cast<uint32_t>(q4 * 32) << 16;
      tmem_ld16(tmem + lanes + kColO + 48 * t, da);
      tmem_ld16(tmem + lanes + kColO + 48 * t + 16, db);
      tmem_ld16(tmem + lanes + kColO + 48 * t + 32, dc);
      tmem_wait_ld();
      const float *st_t = stats + t * 24;
      float wsc_h[G];
#pragma unroll
      for (int h = 0; h < G; ++h) wsc_h[h] = st_t[16 + h];
      float ml0 = 0.0f, ml1 = 0.0f;
      if (tid < G) {
        ml0 = st_t[tid];
        ml1 = st_t[8 + tid];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&oempty[t]);
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const int o = static_cast<int32_t>(da[h]) * 16384 + static_cast<int32_t>(db[h]) * 128 +
                      static_cast<int32_t>(dc[h]);
        const size_t hq = static_cast<size_t>(b) * Hq + g * G + h;
        ws.part_o[(hq * P + p) * kHd + d] = __fmul_rn(static_cast<float>(o), wsc_h[h]);
      }
      if (tid < G) {
        const size_t hq = static_cast<size_t>(b) * Hq + g * G + tid;
        ws.part_ml[(hq * P + p) * 2 + 0] = ml0;
        ws.part_ml[(hq * P + p) * 2 + 1] = ml1;
      }
      ++k;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols) : "memory");
}


// Merge of the persistent kernel's partials, one CTA per row: per head M = max m_p,
// w_p = exp(m_p - M), L = sum w_p l_p, O = sum w_p o_p (partition order), out = dtype(O / L),
// then the row's int8 quantization for o_proj. Same arithmetic as merge_epilogue. The kernel
// is one latency chain, so it is laid out for overlap: each thread first issues its partial
// loads (float4, the first CH partitions of its 4 values); the Hq x P exponentials run one per
// thread; only the partition-order sums (L per head, O per value) are sequential.
constexpr int kMergeThreads = 1024;
template <typename T, int VPT>  // VPT: 4-value vectors of the row per thread
__global__ void __launch_bounds__(kMergeThreads)
    attn_merge_rows_kernel(DecodeWs ws, const int32_t *__restrict__ context_lens, int Hq, int P,
                           T *__restrict__ out, int8_t *__restrict__ out_q,
                           float *__restrict__ out_s) {
  constexpr int CH = VPT == 1 ? 8 : 4;  // partitions whose partials are loaded up front
  griddep_launch();  // the next kernel may start its prologue
  griddep_wait();    // launched with programmatic serialization
  extern __shared__ float msm[];  // W [Hq][P] weights, WL [Hq][P] w * l, L [Hq]
  __shared__ float red[32];
  const int b = blockIdx.x, tid = threadIdx.x;
  const int np = (context_lens[b] + kPart - 1) / kPart;
  const int nv4 = Hq * (kHd / 4);
  const float *mlb = ws.part_ml + static_cast<size_t>(b) * Hq * P * 2;
  const float *pob = ws.part_o + static_cast<size_t>(b) * Hq * P * kHd;
  float4 x[VPT][CH];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int i4 = tid + j * kMergeThreads, h = i4 / (kHd / 4), d = 4 * (i4 % (kHd / 4));
#pragma unroll
    for (int q = 0; q < CH; ++q)
      x[j][q] = (i4 < nv4 && q < np)
                    ? *reinterpret_cast<const float4 *>(pob + (static_cast<size_t>(h) * P + q) * kHd + d)
                    : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  }
  float *W = msm, *WL = msm + Hq * P, *Lh = msm + 2 * Hq * P;
  for (int t = tid; t < Hq * P; t += kMergeThreads) {
    const int h = t / P, q = t - (t / P) * P;
    if (q < np) {
      const float *ml = mlb + static_cast<size_t>(h) * P * 2;
      float M = -__int_as_float(0x7f800000);
      for (int r = 0; r < np; ++r) M = fmaxf(M, ml[2 * r]);
      const float w = exp_s8b(__fsub_rn(ml[2 * q], M));
      W[t] = w;
      WL[t] = __fmul_rn(w, ml[2 * q + 1]);
    }
  }
  __syncthreads();
  for (int h = tid; h < Hq; h += kMergeThreads) {
    float Ls = 0.0f;
    for (int q = 0; q < np; ++q) Ls = __fadd_rn(Ls, WL[h * P + q]);
    Lh[h] = Ls;
  }
  __syncthreads();
  float v[VPT][4];
  float amax = 0.0f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int i4 = tid + j * kMergeThreads, h = i4 / (kHd / 4), d = 4 * (i4 % (kHd / 4));
    if (i4 < nv4) {
      const float *wh = W + h * P;
      float O[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int q = 0; q < CH; ++q) {
        if (q < np) {
          const float wq = wh[q];
          O[0] = __fadd_rn(O[0], __fmul_rn(wq, x[j][q].x));
          O[1] = __fadd_rn(O[1], __fmul_rn(wq, x[j][q].y));
          O[2] = __fadd_rn(O[2], __fmul_rn(wq, x[j][q].z));
          O[3] = __fadd_rn(O[3], __fmul_rn(wq, x[j][q].w));
        }
      }
      for (int q = CH; q < np; ++q) {
        const float4 xq = *reinterpret_cast<const float4 *>(pob + (static_cast<size_t>(h) * P + q) * kHd + d);
        const float wq = wh[q];
        O[0] = __fadd_rn(O[0], __fmul_rn(wq, xq.x));
        O[1] = __fadd_rn(O[1], __fmul_rn(wq, xq.y));
        O[2] = __fadd_rn(O[2], __fmul_rn(wq, xq.z));
        O[3] = __fadd_rn(O[3], __fmul_rn(wq, xq.w));
      }
      const float L = Lh[h];
      T o4[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        v[j][c] = round_to<T>(__fdiv_rn(O[c], L));
        o4[c] = from_f32<T>(v[j][c]);
        amax = fmaxf(amax, fabsf(v[j][c]));
      }
      *reinterpret_cast<uint2 *>(out + static_cast<size_t>(b) * nv4 * 4 + 4 * i4) =
          *reinterpret_cast<const uint2 *>(o4);
    }
  }
  if (!out_q) return;
  amax = block_max(amax, red);
  const QParams qp = qparams(amax, 127.0f);
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int i4 = tid + j * kMergeThreads;
    if (i4 < nv4) {
      char4 c;
      c.x = static_cast<signed char>(qcode(v[j][0], qp.inv, 127));
      c.y = static_cast<signed char>(qcode(v[j][1], qp.inv, 127));
      c.z = static_cast<signed char>(qcode(v[j][2], qp.inv, 127));
      c.w = static_cast<signed char>(qcode(v[j][3], qp.inv, 127));
      *reinterpret_cast<char4 *>(out_q + static_cast<size_t>(b) * nv4 * 4 + 4 * i4) = c;
    }
  }
  if (tid == 0) out_s[b] = qp.scale;
}

inline int num_parts(int max_ctx) { return (max_ctx + kPart - 1) / kPart; }

// 0: persistent tensor-core kernel where the shape allows it, else the per-partition
// tensor-core kernel (default); 1: CUDA-core partition kernel; 2: per-partition tensor-core
int g_attn_impl = 0;

constexpr size_t kStatusBytes = 256;  // the status word, padded to keep the counters aligned

size_t counter_words(int B, int Hq) {
  return static_cast<size_t>(B) * Hq + static_cast<size_t>(B);
}

// status region + completion counters, rounded to 256 bytes
size_t counters_bytes(int B, int Hq) {
  return kStatusBytes + (counter_words(B, Hq) * 4 + 255) / 256 * 256;
}

size_t part_bytes(int B, int Hq, int max_ctx) {
  const size_t P = num_parts(max_ctx);
  return counters_bytes(B, Hq) + static_cast<size_t>(B) * Hq * P * (kHd + 2) * sizeof(float);
}

DecodeWs carve_ws(void *base, int B, int Hq, int max_ctx) {
  uint8_t *p = static_cast<uint8_t *>(base);
  const size_t P = num_parts(max_ctx);
  DecodeWs w;
  w.status = reinterpret_cast<int32_t *>(p);
  w.cnt_group = reinterpret_cast<int32_t *>(p + kStatusBytes);
  w.cnt_row = w.cnt_group + static_cast<size_t>(B) * Hq;
  w.part_o = reinterpret_cast<float *>(p + counters_bytes(B, Hq));
  w.part_ml = w.part_o + static_cast<size_t>(B) * Hq * P * kHd;
  return w;
}

// The persistent kernel + row merge, when the shape allows it: blocks of >= 8 tokens (each
// TMA box then starts on a 1024-byte swizzle atom), 16-byte aligned scale arrays (16-byte
// cp.async), B <= 1024 rows, Hq <= 64 and the merge's (m, l) pairs within 96 KB of shared
// memory, and K/V buffers whose allocation extent the driver reports (the tensor maps cover
// exactly that). Returns 1 when not applicable.
template <typename T>
int launch_persistent(const int8_t *q_i8, const float *q_s, const int8_t *kc, const float *ks,
                      const int8_t *vc, const float *vs, const int32_t *block_table,
                      const int32_t *context_lens, void *out, int8_t *out_q, float *out_s, int B,
                      int Hq, int Hkv, int bs, int bs_log2, int max_blocks, int P, float scale,
                      const DecodeWs &w, int early, cudaStream_t st,
                      const int32_t *row_blocks = nullptr, int NB = 0) {
  const int G = Hq / Hkv;
  if (row_blocks == nullptr) NB = B;
  const size_t merge_smem = 4 * (2 * static_cast<size_t>(Hq) * P + Hq);
  if (bs < 8 || B > pk::kMaxRows || Hq * kHd > kMergeThreads * 8 || merge_smem > 96 * 1024 ||
      !aligned(out, 8) || !aligned(out_q, 4) ||
      !aligned(ks, 16) || !aligned(vs, 16) || !aligned(q_i8, 16))
    return 1;
  const size_t kb = tc::bytes_to_alloc_end(kc), vb = tc::bytes_to_alloc_end(vc);
  const uint64_t rows_k = kb / kHd, rows_v = vb / kHd;
  if (rows_k < static_cast<uint64_t>(bs) || rows_v < static_cast<uint64_t>(bs) ||
      rows_k > 0xffffffffull || rows_v > 0xffffffffull)
    return 1;
  CUtensorMap mk, mv, mq, mk4, mv4;
  if (tc::make_map_2d(&mk, kc, kHd, rows_k, kHd, kHd, bs) ||
      tc::make_map_2d(&mv, vc, kHd, rows_v, kHd, kHd, bs) ||
      tc::make_map_2d(&mq, q_i8, kHd, static_cast<uint64_t>(B) * Hq, kHd, kHd, G))
    return 1;
  // 4-D maps for partitions on consecutive blocks: whole blocks of all heads within the
  // allocation; without them (too small, or an encode failure) every unit takes 2-D copies
  const int nbu = kPart / bs;
  const uint64_t nb_k = rows_k / (static_cast<uint64_t>(bs) * Hkv);
  const uint64_t nb_v = rows_v / (static_cast<uint64_t>(bs) * Hkv);
  const int runs = nb_k >= static_cast<uint64_t>(nbu) && nb_v >= static_cast<uint64_t>(nbu) &&
                   tc::make_map_kv4(&mk4, kc, bs, Hkv, nb_k, nbu) == S8B_OK &&
                   tc::make_map_kv4(&mv4, vc, bs, Hkv, nb_v, nbu) == S8B_OK;
  if (!runs) {
    mk4 = mk;
    mv4 = mv;
  }
  const long U = static_cast<long>(NB) * Hkv * P;
  const int grid = static_cast<int>(U < tc::sm_count() ? U : tc::sm_count());
  // The early loads shorten a decode step's start, but the kernel that carries them streams
  // its steady state slower than attn_persistent_stream_kernel: they pay off only while a CTA
  // has few units to stream (batch 16: 3.25 against 3.31 ms per step; batch 64, 31 units per
  // CTA: 4.98 against 4.95 ms).
  const bool early_ok = early && U <= 16L * grid;
  switch (G) {
#define S8B_PK_CASE(GG)                                                                        \
  case GG: {                                                                                   \
    if (row_blocks != nullptr) {                                                               \
      auto kern = attn_persistent_kernel<T, GG, 16 / GG, false>;                                \
      ensure_smem(reinterpret_cast<const void *>(kern), pk::kSmemRows);                         \
      launch_pdl(kern, grid, pk::kThreads, pk::kSmemRows, st, mk, mv, mq, mk4, mv4, runs, q_s,  \
                 ks, vs, block_table, context_lens, B, Hq, Hkv, bs_log2, max_blocks, P, scale,  \
                 w, 0, q_i8, row_blocks, NB);                                                   \
    } else {                                                                                   \
      if (early_ok) {                                                                          \
        auto kern = attn_persistent_kernel<T, GG, 1, true>;                                     \
        ensure_smem(reinterpret_cast<const void *>(kern), pk::kSmem);                           \
        launch_pdl(kern, grid, pk::kThreads, pk::kSmem, st, mk, mv, mq, mk4, mv4, runs, q_s,    \
                   ks, vs, block_table, context_lens, B, Hq, Hkv, bs_log2, max_blocks, P,       \
                   scale, w, 1, q_i8, row_blocks, NB);                                          \
      } else if (GG <= 5) {                                                                    \
        auto kern = attn_persistent_stream_kernel<T, GG>;                                       \
        ensure_smem(reinterpret_cast<const void *>(kern), pk::kSmem);                           \
        launch_pdl(kern, grid, pk::kThreads, pk::kSmem, st, mk, mv, mq, mk4, mv4, runs, q_s,    \
                   ks, vs, block_table, context_lens, B, Hq, Hkv, bs_log2, max_blocks, P,       \
                   scale, w);                                                                   \
      } else {                                                                                 \
        auto kern = attn_persistent_kernel<T, GG, 1, false>;                                    \
        ensure_smem(reinterpret_cast<const void *>(kern), pk::kSmem);                           \
        launch_pdl(kern, grid, pk::kThreads, pk::kSmem, st, mk, mv, mq, mk4, mv4, runs, q_s,    \
                   ks, vs, block_table, context_lens, B, Hq, Hkv, bs_log2, max_blocks, P,       \
                   scale, w, 0, q_i8, row_blocks, NB);                                          \
      }                                                                                        \
    }                                                                                          \
    break;                                                                                     \
  }
    S8B_PK_CASE(1)
    S8B_PK_CASE(2)
    S8B_PK_CASE(3)
    S8B_PK_CASE(4)
    S8B_PK_CASE(5)
    S8B_PK_CASE(6)
    S8B_PK_CASE(7)
    S8B_PK_CASE(8)
#undef S8B_PK_CASE
    default:
      return S8B_ERR_SHAPE;
  }
  const int vpt = (Hq * kHd / 4 + kMergeThreads - 1) / kMergeThreads;
  auto merge = vpt <= 1 ? attn_merge_rows_kernel<T, 1> : attn_merge_rows_kernel<T, 2>;
  ensure_smem(reinterpret_cast<const void *>(merge), 96 * 1024);
  launch_pdl(merge, B, kMergeThreads, merge_smem, st, w, context_lens, Hq, P,
             static_cast<T *>(out), out_q, out_s);
  return check_launch(2);
}

template <typename T>
int launch_decode(const int8_t *q_i8, const float *q_s, const int8_t *kc, const float *ks,
                  const int8_t *vc, const float *vs, const int32_t *block_table,
                  const int32_t *context_lens, void *out, int8_t *out_q, float *out_s, int B,
                  int Hq, int Hkv, int bs, int max_blocks, int max_ctx, float scale,
                  void *workspace, cudaStream_t st, int early = 0,
                  const int32_t *row_blocks = nullptr, int NB = 0) {
  const int P = num_parts(max_ctx);
  const int G = Hq / Hkv;
  int bs_log2 = 0;
  while ((1 << bs_log2) < bs) ++bs_log2;
  const DecodeWs w = carve_ws(workspace, B, Hq, max_ctx);
  if (g_attn_impl == 0) {
    const int rc = launch_persistent<T>(q_i8, q_s, kc, ks, vc, vs, block_table, context_lens, out,
                                        out_q, out_s, B, Hq, Hkv, bs, bs_log2, max_blocks, P,
                                        scale, w, early, st, row_blocks, NB);
    if (rc != 1) return rc;
  }
  // The partition kernels count completions; their counters start from zero on every launch.
  const cudaError_t ce = cudaMemsetAsync(w.cnt_group, 0, counter_words(B, Hq) * 4, st);
  if (ce != cudaSuccess) {
    record_cuda_error(ce);
    return S8B_ERR_CUDA;
  }
  if (g_attn_impl != 1) {
    switch (G) {
#define S8B_TC_CASE(GG)                                                                        \
  case GG: {                                                                                   \
    auto kern = attn_partition_tc_kernel<T, GG>;                                                \
    ensure_smem(reinterpret_cast<const void *>(kern), TcPartSmem<GG>::bytes);                   \
    kern<<<dim3(P, Hkv, B), kTcThreads, TcPartSmem<GG>::bytes, st>>>(                           \
        q_i8, q_s, kc, ks, vc, vs, block_table, context_lens, Hq, Hkv, bs_log2, max_blocks, P,  \
        scale, w, static_cast<T *>(out), out_q, out_s);                                         \
    return check_launch(1);                                                                    \
  }
      S8B_TC_CASE(1)
      S8B_TC_CASE(2)
      S8B_TC_CASE(3)
      S8B_TC_CASE(4)
      S8B_TC_CASE(5)
      S8B_TC_CASE(6)
      S8B_TC_CASE(7)
      S8B_TC_CASE(8)
#undef S8B_TC_CASE
      default:
        return S8B_ERR_SHAPE;
    }
  }
  switch (G) {
#define S8B_PART_CASE(GG)                                                                      \
  case GG: {                                                                                   \
    auto kern = attn_partition_kernel<T, GG>;                                                   \
    ensure_smem(reinterpret_cast<const void *>(kern), PartSmem<GG>::bytes);                     \
    kern<<<dim3(P, Hkv, B), kPartThreads, PartSmem<GG>::bytes, st>>>(                           \
        q_i8, q_s, kc, ks, vc, vs, block_table, context_lens, Hq, Hkv, bs_log2, max_blocks, P,  \
        scale, w, static_cast<T *>(out), out_q, out_s);                                         \
    break;                                                                                     \
  }
    S8B_PART_CASE(1)
    S8B_PART_CASE(2)
    S8B_PART_CASE(3)
    S8B_PART_CASE(4)
    S8B_PART_CASE(5)
    S8B_PART_CASE(6)
    S8B_PART_CASE(7)
    S8B_PART_CASE(8)
#undef S8B_PART_CASE
    default:
      return S8B_ERR_SHAPE;
  }
  return check_launch(1);
}

int check_attn_shape(int B, int Hq, int Hkv, int D, int bs, int max_blocks, int max_ctx) {
  if (B < 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0 || Hq / Hkv > 8 || D != kHd)
    return S8B_ERR_SHAPE;
  if (bs <= 0 || (bs & (bs - 1)) != 0 || kPart % bs != 0 || max_ctx <= 0 ||
      max_blocks * bs < max_ctx)
    return S8B_ERR_SHAPE;
  if (num_parts(max_ctx) * Hq > 8192) return S8B_ERR_SHAPE;  // combine smem bound
  return S8B_OK;
}

}  // namespace
}  // namespace s8b

using namespace s8b;

namespace s8b {
namespace {
template <typename T>
int launch_qkv_post(RowSrc<T> src, const int32_t *positions, const float *cos_tab,
                    const float *sin_tab, const void *q_norm_w, const void *k_norm_w, float eps,
                    int M, int Hq, int Hkv, int8_t *q_i8, float *q_s, void *q_out, int8_t *kc,
                    float *ks, int8_t *vc, float *vs, const int32_t *slot_mapping,
                    const int32_t *block_table, int max_blocks, int block_size, void *stream) {
  launch_pdl(qkv_post_kernel<T>, dim3((Hq + 2 * Hkv + kQkvWarps - 1) / kQkvWarps, M),
             kQkvWarps * 32, 0, (cudaStream_t)stream, src, positions, cos_tab, sin_tab,
             static_cast<const T *>(q_norm_w), static_cast<const T *>(k_norm_w), eps, Hq, Hkv,
             q_i8, q_s, static_cast<T *>(q_out), kc, ks, vc, vs, slot_mapping, block_table,
             max_blocks, block_size);
  return check_launch();
}

int check_qkv_post(const int32_t *positions, const float *cos_tab, const float *sin_tab,
                   int max_pos, const void *q_norm_w, const void *k_norm_w, int M, int Hq,
                   int Hkv, int D, int8_t *q_i8, float *q_s, int8_t *kc, float *ks, int8_t *vc,
                   float *vs, const int32_t *slot_mapping, const int32_t *block_table,
                   int block_size) {
  if (!positions || !cos_tab || !sin_tab || !q_norm_w || !k_norm_w || !q_i8 || !q_s || !kc ||
      !ks || !vc || !vs || (!slot_mapping && !block_table))
    return S8B_ERR_ARG;
  if (M < 0 || M > 65535 || D != kHd || Hq <= 0 || Hkv <= 0 || block_size <= 0 || max_pos <= 0)
    return S8B_ERR_SHAPE;
  if (!aligned(q_i8, 16) || !aligned(kc, 16) || !aligned(vc, 16)) return S8B_ERR_ALIGN;
  return S8B_OK;
}
}  // namespace
}  // namespace s8b

extern "C" int s8b_qkv_post(const void *qkv, const int32_t *positions, const float *cos_tab,
                            const float *sin_tab, int max_pos, const void *q_norm_w,
                            const void *k_norm_w, float eps, int M, int Hq, int Hkv, int D,
                            int8_t *q_i8, float *q_s, void *q_out, int8_t *kc, float *ks,
                            int8_t *vc, float *vs, const int32_t *slot_mapping,
                            const int32_t *block_table, int max_blocks, int block_size,
                            int dtype, void *stream) {
  if (!qkv) return S8B_ERR_ARG;
  const int e = check_qkv_post(positions, cos_tab, sin_tab, max_pos, q_norm_w, k_norm_w, M, Hq,
                               Hkv, D, q_i8, q_s, kc, ks, vc, vs, slot_mapping, block_table,
                               block_size);
  if (e) return e;
  if (!aligned(qkv, 8)) return S8B_ERR_ALIGN;
  if (M == 0) return S8B_OK;
  S8B_DISPATCH_DTYPE(dtype, T,
                     return launch_qkv_post<T>(row_src<T>(qkv, (Hq + 2 * Hkv) * kHd), positions,
                                               cos_tab, sin_tab, q_norm_w, k_norm_w, eps, M, Hq,
                                               Hkv, q_i8, q_s, q_out, kc, ks, vc, vs,
                                               slot_mapping, block_table, max_blocks,
                                               block_size, stream));
}

extern "C" int s8b_qkv_post_split(const int32_t *part, int C, const float *xs, const float *ws,
                                  const int32_t *positions, const float *cos_tab,
                                  const float *sin_tab, int max_pos, const void *q_norm_w,
                                  const void *k_norm_w, float eps, int M, int Hq, int Hkv, int D,
                                  int8_t *q_i8, float *q_s, void *q_out, int8_t *kc, float *ks,
                                  int8_t *vc, float *vs, const int32_t *slot_mapping,
                                  const int32_t *block_table, int max_blocks, int block_size,
                                  int dtype, void *stream) {
  if (!part || !xs || !ws) return S8B_ERR_ARG;
  if (C < 1 || C > 8) return S8B_ERR_SHAPE;
  const int e = check_qkv_post(positions, cos_tab, sin_tab, max_pos, q_norm_w, k_norm_w, M, Hq,
                               Hkv, D, q_i8, q_s, kc, ks, vc, vs, slot_mapping, block_table,
                               block_size);
  if (e) return e;
  if (!aligned(part, 16) || !aligned(ws, 16)) return S8B_ERR_ALIGN;
  if (M == 0) return S8B_OK;
  S8B_DISPATCH_DTYPE(dtype, T,
                     return launch_qkv_post<T>(
                         row_src_split<T>(part, C, xs, ws, M, (Hq + 2 * Hkv) * kHd), positions,
                         cos_tab, sin_tab, q_norm_w, k_norm_w, eps, M, Hq, Hkv, q_i8, q_s, q_out,
                         kc, ks, vc, vs, slot_mapping, block_table, max_blocks, block_size,
                         stream));
}

extern "C" int s8b_kv_write_paged(const void *k, const void *v, int8_t *kc, float *ks, int8_t *vc,
                                  float *vs, const int32_t *slot_mapping, int T_, int Hkv, int D,
                                  int block_size, int rotate_k, int dtype, void *stream) {
  if (!k || !v || !kc || !ks || !vc || !vs || !slot_mapping) return S8B_ERR_ARG;
  if (T_ < 0 || Hkv <= 0 || D != kHd || block_size <= 0) return S8B_ERR_SHAPE;
  if (!aligned(kc, 16) || !aligned(vc, 16)) return S8B_ERR_ALIGN;
  if (T_ == 0) return S8B_OK;
  S8B_DISPATCH_DTYPE(dtype, T,
                     kv_write_kernel<T><<<T_, 256, 0, (cudaStream_t)stream>>>(
                         static_cast<const T *>(k), static_cast<const T *>(v), kc, ks, vc, vs,
                         slot_mapping, Hkv, block_size, rotate_k));
  return check_launch();
}

extern "C" size_t s8b_paged_decode_workspace_size(int B, int Hq, int D, int max_ctx) {
  (void)D;
  return part_bytes(B, Hq, max_ctx);
}

namespace {
int paged_decode_q8(const int8_t *q_i8, const float *q_s, const int8_t *kc, const float *ks,
                    const int8_t *vc, const float *vs, const int32_t *block_table,
                    const int32_t *context_lens, void *out, int8_t *out_q, float *out_s, int B,
                    int Hq, int Hkv, int D, int block_size, int max_blocks, int max_ctx,
                    float scale, void *workspace, size_t workspace_bytes, int dtype,
                    void *stream, int early) {
  if (!q_i8 || !q_s || !kc || !ks || !vc || !vs || !block_table || !context_lens || !out ||
      ((out_q == nullptr) != (out_s == nullptr)))
    return S8B_ERR_ARG;
  const int e = check_attn_shape(B, Hq, Hkv, D, block_size, max_blocks, max_ctx);
  if (e) return e;
  if (!aligned(q_i8, 16) || !aligned(kc, 16) || !aligned(vc, 16)) return S8B_ERR_ALIGN;
  if (!workspace || workspace_bytes < part_bytes(B, Hq, max_ctx)) return S8B_ERR_WORKSPACE;
  if (B == 0) return S8B_OK;
  S8B_DISPATCH_DTYPE(dtype, T,
                     return launch_decode<T>(q_i8, q_s, kc, ks, vc, vs, block_table,
                                             context_lens, out, out_q, out_s, B, Hq, Hkv,
                                             block_size, max_blocks, max_ctx, scale,
                                             static_cast<float *>(workspace),
                                             (cudaStream_t)stream, early));
}
}  // namespace

extern "C" int s8b_paged_decode_q8(const int8_t *q_i8, const float *q_s, const int8_t *kc,
                                   const float *ks, const int8_t *vc, const float *vs,
                                   const int32_t *block_table, const int32_t *context_lens,
                                   void *out, int8_t *out_q, float *out_s, int B, int Hq, int Hkv,
                                   int D, int block_size, int max_blocks, int max_ctx,
                                   float scale, void *workspace, size_t workspace_bytes,
                                   int dtype, void *stream) {
  return paged_decode_q8(q_i8, q_s, kc, ks, vc, vs, block_table, context_lens, out, out_q, out_s,
                         B, Hq, Hkv, D, block_size, max_blocks, max_ctx, scale, workspace,
                         workspace_bytes, dtype, stream, 0);
}

extern "C" int s8b_paged_decode_q8_step(const int8_t *q_i8, const float *q_s, const int8_t *kc,
                                        const float *ks, const int8_t *vc, const float *vs,
                                        const int32_t *block_table,
                                        const int32_t *context_lens, void *out, int8_t *out_q,
                                        float *out_s, int B, int Hq, int Hkv, int D,
                                        int block_size, int max_blocks, int max_ctx, float scale,
                                        void *workspace, size_t workspace_bytes, int dtype,
                                        void *stream) {
  return paged_decode_q8(q_i8, q_s, kc, ks, vc, vs, block_table, context_lens, out, out_q, out_s,
                         B, Hq, Hkv, D, block_size, max_blocks, max_ctx, scale, workspace,
                         workspace_bytes, dtype, stream, 1);
}

extern "C" int s8b_paged_prefill_block_rows(int Hq, int Hkv) {
  if (Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0 || Hq / Hkv > 8) return S8B_ERR_SHAPE;
  return 16 / (Hq / Hkv);
}

extern "C" int s8b_paged_prefill_q8(const int8_t *q_i8, const float *q_s, const int8_t *kc,
                                    const float *ks, const int8_t *vc, const float *vs,
                                    const int32_t *block_table, const int32_t *context_lens,
                                    const int32_t *row_blocks, int n_row_blocks, void *out,
                                    int8_t *out_q, float *out_s, int B, int Hq, int Hkv, int D,
                                    int block_size, int max_blocks, int max_ctx, float scale,
                                    void *workspace, size_t workspace_bytes, int dtype,
                                    void *stream) {
  if (!q_i8 || !q_s || !kc || !ks || !vc || !vs || !block_table || !context_lens || !out ||
      (n_row_blocks > 0 && !row_blocks) || ((out_q == nullptr) != (out_s == nullptr)))
    return S8B_ERR_ARG;
  const int e = check_attn_shape(B, Hq, Hkv, D, block_size, max_blocks, max_ctx);
  if (e) return e;
  if (n_row_blocks < 0 || n_row_blocks > B) return S8B_ERR_SHAPE;
  if (!aligned(q_i8, 16) || !aligned(kc, 16) || !aligned(vc, 16)) return S8B_ERR_ALIGN;
  if (!workspace || workspace_bytes < part_bytes(B, Hq, max_ctx)) return S8B_ERR_WORKSPACE;
  if (B == 0) return S8B_OK;
  // without row blocks (or where the persistent kernel does not apply) every row is its own
  // unit, as in s8b_paged_decode_q8
  S8B_DISPATCH_DTYPE(dtype, T,
                     return launch_decode<T>(q_i8, q_s, kc, ks, vc, vs, block_table,
                                             context_lens, out, out_q, out_s, B, Hq, Hkv,
                                             block_size, max_blocks, max_ctx, scale,
                                             static_cast<float *>(workspace),
                                             (cudaStream_t)stream, 0,
                                             n_row_blocks > 0 ? row_blocks : nullptr,
                                             n_row_blocks));
}

// ---------------------------------------------------------- no-allocation variant ----
// Scratch for s8b_paged_decode_q8_noalloc: the per-partition partial sums live in this
// fixed device array instead of a caller workspace. Every GPU that loads the library holds
// it until the process exits. Host code must not pass `g_decode_static_scratch` itself to a
// kernel: on the host that name is only a stand-in for the device symbol, so its device
// address is looked up once per device with cudaGetSymbolAddress.
constexpr size_t kStaticScratchBytes = size_t(16) << 20;  // 16 MiB
static __device__ __align__(256) float g_decode_static_scratch[kStaticScratchBytes / sizeof(float)];

namespace {
std::mutex g_static_scratch_mu;
std::map<int, float *> g_static_scratch_addr;  // device ordinal -> device address

// Runs on the calling thread's current device; the first call per device does the lookup.
int static_scratch_address(float **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    record_cuda_error(e);
    return S8B_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lk(g_static_scratch_mu);
  auto it = g_static_scratch_addr.find(dev);
  if (it == g_static_scratch_addr.end()) {
    float *p = nullptr;
    e = cudaGetSymbolAddress(reinterpret_cast<void **>(&p), g_decode_static_scratch);
    if (e != cudaSuccess || p == nullptr) {
      record_cuda_error(e);
      return S8B_ERR_CUDA;
    }
    it = g_static_scratch_addr.emplace(dev, p).first;
  }
  *out = it->second;
  return S8B_OK;
}
}  // namespace

extern "C" int s8b_paged_decode_q8_noalloc(const int8_t *q_i8, const float *q_s, const int8_t *kc,
                                           const float *ks, const int8_t *vc, const float *vs,
                                           const int32_t *block_table,
                                           const int32_t *context_lens, void *out, int8_t *out_q,
                                           float *out_s, int B, int Hq, int Hkv, int D,
                                           int block_size, int max_blocks, int max_ctx,
                                           float scale, int dtype, void *stream) {
  if (!q_i8 || !q_s || !kc || !ks || !vc || !vs || !block_table || !context_lens || !out ||
      ((out_q == nullptr) != (out_s == nullptr)))
    return S8B_ERR_ARG;
  const int e = check_attn_shape(B, Hq, Hkv, D, block_size, max_blocks, max_ctx);
  if (e) return e;
  if (!aligned(q_i8, 16) || !aligned(kc, 16) || !aligned(vc, 16)) return S8B_ERR_ALIGN;
  if (part_bytes(B, Hq, max_ctx) > kStaticScratchBytes) return S8B_ERR_SCRATCH_LIMIT;
  if (dtype != S8B_BF16 && dtype != S8B_FP16) return S8B_ERR_DTYPE;
  if (B == 0) return S8B_OK;
  float *part = nullptr;
  const int rc = static_scratch_address(&part);
  if (rc) return rc;
  // The array is laid out like a caller workspace: the status word at byte 0 (sticky until
  // s8b_paged_decode_noalloc_status replaces it), the completion counters, which launch_decode
  // zeroes before every launch of the kernels that use them, then the partition partials,
  // which are fully written before anything reads them.
  S8B_DISPATCH_DTYPE(dtype, T,
                     return launch_decode<T>(q_i8, q_s, kc, ks, vc, vs, block_table,
                                             context_lens, out, out_q, out_s, B, Hq, Hkv,
                                             block_size, max_blocks, max_ctx, scale, part,
                                             (cudaStream_t)stream));
}

extern "C" int s8b_paged_decode_noalloc_status(int32_t *previous, int32_t replace_with) {
  if (!previous) return S8B_ERR_ARG;
  float *part = nullptr;
  const int rc = static_scratch_address(&part);
  if (rc) return rc;
  // Plain synchronous copies of one word: they wait for the device's earlier work on the
  // legacy default stream and allocate nothing.
  cudaError_t e = cudaMemcpy(previous, part, sizeof(int32_t), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) e = cudaMemcpy(part, &replace_with, sizeof(int32_t), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    record_cuda_error(e);
    return S8B_ERR_CUDA;
  }
  return S8B_OK;
}

extern "C" size_t s8b_paged_decode_ref_workspace_size(int B, int Hq, int D, int max_ctx) {
  const size_t part = (part_bytes(B, Hq, max_ctx) + 255) / 256 * 256;
  const size_t q = (static_cast<size_t>(B) * Hq * D + 255) / 256 * 256;
  const size_t qs = (static_cast<size_t>(B) * Hq * sizeof(float) + 255) / 256 * 256;
  return part + q + qs;
}

extern "C" int s8b_paged_decode(const void *q, const int8_t *kc, const float *ks, const int8_t *vc,
                                const float *vs, const int32_t *block_table,
                                const int32_t *context_lens, void *out, int B, int Hq, int Hkv,
                                int D, int block_size, int max_blocks, int max_ctx, float scale,
                                void *workspace, size_t workspace_bytes, int dtype, void *stream) {
  if (!q || !out) return S8B_ERR_ARG;
  const int e = check_attn_shape(B, Hq, Hkv, D, block_size, max_blocks, max_ctx);
  if (e) return e;
  if (!workspace || workspace_bytes < s8b_paged_decode_ref_workspace_size(B, Hq, D, max_ctx))
    return S8B_ERR_WORKSPACE;
  if (!aligned(workspace, 256)) return S8B_ERR_ALIGN;
  if (B == 0) return S8B_OK;
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  float *part = reinterpret_cast<float *>(ws);
  int8_t *q8 = reinterpret_cast<int8_t *>(ws + (part_bytes(B, Hq, max_ctx) + 255) / 256 * 256);
  float *qsc = reinterpret_cast<float *>(q8 + (static_cast<size_t>(B) * Hq * D + 255) / 256 * 256);
  cudaStream_t st = (cudaStream_t)stream;
  S8B_DISPATCH_DTYPE(dtype, T, {
    q_rotate_quant_kernel<T><<<B, 256, 0, st>>>(static_cast<const T *>(q), Hq, q8, qsc);
    check_launch(1);
    return launch_decode<T>(q8, qsc, kc, ks, vc, vs, block_table, context_lens, out, nullptr,
                            nullptr, B, Hq, Hkv, block_size, max_blocks, max_ctx, scale, part, st);
  });
}

extern "C" size_t s8b_paged_decode_status_offset(int B, int Hq) {
  (void)B;
  (void)Hq;
  return 0;  // the same word for every shape (see carve_ws)
}

extern "C" int s8b_set_attention_impl(int impl) {
  if (impl < 0 || impl > 2) return S8B_ERR_ARG;
  s8b::g_attn_impl = impl;
  return S8B_OK;
}
