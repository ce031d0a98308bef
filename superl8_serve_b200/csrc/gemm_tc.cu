// W8A8 GEMM on the 5th-generation tensor cores (tcgen05.mma kind::i8) for decode token counts
// that make the contraction dense enough (16..256 tokens per launch).
//
// Shape: y[m, n] = dequant( sum_k xq[m, k] * w[n, k] ). The MMA is issued "swap-AB":
// A = 128 weight rows x 32 K-bytes, B = NT tokens x 32 K-bytes, D = 128 x NT int32 in TMEM,
// so the weight matrix (the HBM stream) fills the 128-row MMA dimension and the small token
// count is the N dimension.
//
// Work split: thread-block clusters of C CTAs walk the 128-row weight tiles; the C CTAs of a
// cluster split each tile's K range and reduce their int32 partial tiles through distributed
// shared memory (see gemm_tc_kernel). Launched with programmatic stream serialization: the
// first weight tiles stream in while the preceding kernel finishes.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <map>
#include <mutex>

#include "common.cuh"
#include "tcgen05.cuh"

namespace s8b {
namespace {

using namespace tc;

constexpr int kBM = 128;          // weight rows per tile (MMA M)
constexpr int kBK = 128;          // K bytes per stage (one 128B swizzle atom row)
constexpr int kABytes = kBM * kBK;
constexpr int kThreads = 320;
constexpr int kEpi = 256;  // epilogue threads: two warps per TMEM lane quadrant
constexpr int kMaxStages = 8;
constexpr int kSmemBudget = 220 * 1024;

struct TcSmemHeader {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t recv;     // split-K: receive buffer filled by every CTA of the cluster (tx bytes)
  uint64_t done;     // split-K: every CTA of the cluster finished reducing its receive buffer
  uint32_t tmem_base;
  int abort;
  float xs[256];     // per-token activation scales of this launch's token tile
  float wsc[2][128];  // per-row weight scales of the tile in each TMEM buffer
};

// Pack W [N, K] (row-major int8) into unit images: unit (tile, kc) holds rows
// tile*128..+127, bytes kc*128..+127 as the 128B-swizzled K-major shared-memory image
// (16-byte chunk c of row r stored at chunk c ^ (r % 8)); rows beyond N are zero.
__global__ void pack_tc_kernel(const int8_t *__restrict__ w, int N, int K,
                               int8_t *__restrict__ packed) {
  const int kc = K / kBK;
  const size_t chunks = static_cast<size_t>((N + kBM - 1) / kBM) * kc * kBM * 8;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < chunks;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i & 7);
    const int r = static_cast<int>((i >> 3) % kBM);
    const size_t unit = (i >> 3) / kBM;
    const int tile = static_cast<int>(unit / kc), kk = static_cast<int>(unit % kc);
    const int n = tile * kBM + r;
    int4 v = make_int4(0, 0, 0, 0);
    if (n < N) v = *reinterpret_cast<const int4 *>(w + static_cast<size_t>(n) * K + kk * kBK + c * 16);
    *reinterpret_cast<int4 *>(packed + unit * kABytes + r * kBK + ((c ^ (r & 7)) * 16)) = v;
  }
}

// PARTS: the layout carries the on-chip split-K buffers (cluster reduction, out_kind 0/1).
// Without them (out_kind 2: partials go to global memory) the kernel stays under ~200 KB, so
// a CTA of the small row kernels fits beside it and programmatic dependent launch can start
// it, and its weight prefetch, while the preceding kernel still runs.
constexpr int kLeanBudget = 200 * 1024;
template <int NT, bool PARTS = true>
struct TcLayout {
  static constexpr int kBBytes = NT * kBK;
  static constexpr int kStageBytes = kABytes + kBBytes;
  // split-K buffers (token tiles up to 64 only), rows of NT int32 plus a 16-byte pad
  // (conflict-free row-per-thread access): the staging tile [128 rows] this CTA sends from,
  // and the receive buffer [C source slots][ceil(128/C) rows] (<= 136 rows for C <= 8)
  static constexpr int kPartPitch = NT * 4 + 16;
  static constexpr int kStageRows = (PARTS && NT <= 64) ? kBM : 0;
  static constexpr int kRecvRows = (PARTS && NT <= 64) ? 136 : 0;
  static constexpr int kPartBytes = (kStageRows + kRecvRows) * kPartPitch;
  static constexpr int kBudget = PARTS ? kSmemBudget : kLeanBudget;
  static constexpr int kStages =
      (kBudget - 4096 - kPartBytes) / kStageBytes < kMaxStages
          ? (kBudget - 4096 - kPartBytes) / kStageBytes
          : kMaxStages;
  static constexpr int kTmemCols = 2 * NT < 32 ? 32 : 2 * NT;
  static constexpr size_t kSmem =
      1024 + static_cast<size_t>(kStages) * kStageBytes + kPartBytes + 3072;
};

struct TcArgs {
  const int8_t *wpacked;  // weights pre-packed into shared-memory images (null: TMA 2D path)
  const float *xs;
  const float *ws;
  void *y;
  int32_t *status;  // workspace status word
  int out_kind, M, N, K, m0, n_tiles, kc;
  int csplit;     // CTAs sharing each tile's K range (1: no split)
  int nclusters;  // CTA groups in the grid (launched as clusters unless out_kind == 2)
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t mapa(uint32_t saddr, uint32_t cta) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(cta));
  return r;
}
__device__ __forceinline__ void mbar_arrive_remote(uint64_t *bar, uint32_t cta) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(
                   mapa(smem_u32(bar), cta))
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\nmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait with cluster-scope acquire (peer CTAs arrive on this barrier).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity,
                                                  volatile int *abort, int32_t *status) {
  const uint64_t t0 = now_ns();
  while (!mbar_try_wait_cluster(bar, parity)) {
    if (*abort) return false;
    if (now_ns() - t0 > 2000000000ull) {
      *abort = 1;
      atomicExch(status, S8B_ERR_TIMEOUT);
      return false;
    }
  }
  return true;
}

// W8A8 GEMM on the 5th-generation tensor cores (tcgen05.mma kind::i8), swap-AB: A = 128
// weight rows x 32 K-bytes, B = NT tokens x 32 K-bytes, D = 128 x NT int32 in TMEM, so the
// weight matrix (the HBM stream) fills the 128-row MMA dimension.
//
// Work split. Clusters of C CTAs walk the 128-row weight tiles round-robin; CTA r of a
// cluster streams K chunks [r*kc/C, (r+1)*kc/C) of every tile of its cluster. With C > 1 the
// epilogue stages its int32 partial tile in shared memory and one thread moves each CTA's
// rows (rows [ceil(r*128/C), ceil((r+1)*128/C)) belong to CTA r) into that CTA's receive
// buffer with one shared-to-shared bulk copy, completing on the owner's mbarrier as a byte
// count; the owner then sums the C slots from its own shared memory (integer sums: exact in
// any order), dequantizes and stores. No global workspace, atomics, device-wide fences or
// remote loads. C is chosen per shape by the host to balance the tiles over the clusters.
//
// Roles (320 threads): warp 0 issues the loads (TMA or bulk copies of pre-packed weight
// images; the weight copies of the first stages go out before griddepcontrol.wait, the
// activations after it), warp 1 issues the MMAs (one thread) and owns the TMEM allocation,
// warps 2-9 drain TMEM: warps w and w + 4 share lane quadrant w % 4 and take one half of the
// token columns each. The accumulator is double-buffered in TMEM. Every mbarrier wait is
// bounded: on timeout the kernel records S8B_ERR_TIMEOUT in the status word.
template <typename T, int NT, bool PARTS = true>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_w,
                   const __grid_constant__ CUtensorMap tmap_x, TcArgs a) {
  using Lay = TcLayout<NT, PARTS>;
  constexpr int S = Lay::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *part = smem + static_cast<size_t>(S) * Lay::kStageBytes;
  TcSmemHeader *hdr = reinterpret_cast<TcSmemHeader *>(part + Lay::kPartBytes);
  uint8_t *recvb = part + Lay::kStageRows * Lay::kPartPitch;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C = a.csplit;
  // out_kind 2 stores each CTA's partial tile (no cluster, no on-chip reduction)
  const bool clustered = C > 1 && a.out_kind != 2;
  const uint32_t crank = clustered ? cluster_rank() : static_cast<uint32_t>(blockIdx.x % C);
  const int cid = blockIdx.x / C;
  const int k_lo = static_cast<int>(crank) * a.kc / C, k_hi = (static_cast<int>(crank) + 1) * a.kc / C;
  const int nk = k_hi - k_lo;
  const int my_tiles = cid < a.n_tiles ? (a.n_tiles - 1 - cid) / a.nclusters + 1 : 0;
  const long long n_units = static_cast<long long>(my_tiles) * nk;
  // split-K row ownership: row r of a tile is reduced by CTA (r * C) / 128
  const int r0 = (static_cast<int>(crank) * kBM + C - 1) / C;
  const int r1 = ((static_cast<int>(crank) + 1) * kBM + C - 1) / C;
  const int slot_rows = (kBM + C - 1) / C;
  const uint32_t recv_bytes = static_cast<uint32_t>(C * (r1 - r0) * (NT * 4 + 16));

  griddep_launch();
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&hdr->full[s], 1);
      mbar_init(&hdr->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&hdr->tmem_full[b], 1);
      mbar_init(&hdr->tmem_empty[b], kEpi);
    }
    mbar_init(&hdr->recv, 1);
    mbar_init(&hdr->done, C);
    hdr->abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    if (clustered && my_tiles > 0)  // the first tile's receive buffer: C slots of this CTA's rows
      mbar_expect_tx(&hdr->recv, recv_bytes);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&hdr->tmem_base)),
                 "r"(Lay::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  if (clustered) {  // peers arrive on this CTA's barriers: all must be initialised first
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
  }
  tc_fence_after();
  const uint32_t tmem = hdr->tmem_base;
  volatile int *abort = &hdr->abort;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer ----
    if (lane == 0) {
      if (!a.wpacked)
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_w)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_x)) : "memory");
      // Unit i is (tile cid + (i / nk) * nclusters, K chunk k_lo + i % nk). The (tile, kk)
      // pair advances by a compare and an add: a 64-bit division per unit costs this one
      // thread several hundred nanoseconds, which would pace the whole weight stream.
      struct UnitPos {
        int tile, kk;
      };
      auto advance = [&](UnitPos &u) {
        if (++u.kk == k_hi) {
          u.kk = k_lo;
          u.tile += a.nclusters;
        }
      };
      auto load_a = [&](const UnitPos &u, uint8_t *sa, uint64_t *bar) {
        if (a.wpacked)
          bulk_load(sa, a.wpacked + (static_cast<size_t>(u.tile) * a.kc + u.kk) * kABytes, kABytes,
                    bar);
        else
          tma_load_2d(sa, &tmap_w, u.kk * kBK, u.tile * kBM, bar);
      };
      auto load_b = [&](const UnitPos &u, uint8_t *sa, uint64_t *bar) {
        tma_load_2d(sa + kABytes, &tmap_x, u.kk * kBK, a.m0, bar);
      };
      // weights of the first stages before the previous kernel has finished
      const int pre = n_units < S ? static_cast<int>(n_units) : S;
      UnitPos u{cid, k_lo};
      for (int i = 0; i < pre; ++i, advance(u)) {
        mbar_expect_tx(&hdr->full[i], Lay::kStageBytes);
        load_a(u, smem + static_cast<size_t>(i) * Lay::kStageBytes, &hdr->full[i]);
      }
      griddep_wait();
      {
        UnitPos v{cid, k_lo};
        for (int i = 0; i < pre; ++i, advance(v))
          load_b(v, smem + static_cast<size_t>(i) * Lay::kStageBytes, &hdr->full[i]);
      }
      long long issued = pre;
      int s = pre % S;
      uint32_t ph = pre == S ? 1u : 0u;  // phase parity of stage s's next fill
      for (long long i = pre; i < n_units; ++i, ++issued, advance(u)) {
        if (!mbar_wait(&hdr->empty[s], ph ^ 1, abort, a.status)) break;
        uint8_t *sa = smem + static_cast<size_t>(s) * Lay::kStageBytes;
        mbar_expect_tx(&hdr->full[s], Lay::kStageBytes);
        load_a(u, sa, &hdr->full[s]);
        load_b(u, sa, &hdr->full[s]);
        if (++s == S) {
          s = 0;
          ph ^= 1u;
        }
      }
      if (*abort) {
        // let the copies already issued land before the CTA's shared memory goes away
        const long long first = issued > S ? issued - S : 0;
        for (long long i = first; i < issued; ++i)
          mbar_drain(&hdr->full[i % S], static_cast<uint32_t>((i / S) & 1));
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------- MMA issuer ----
    if (lane == 0) {
      constexpr uint32_t idesc = i8_idesc(kBM, NT);
      int seg = 0, kk = 0, s = 0;  // counters, no per-unit division
      uint32_t ph = 0;
      for (long long i = 0; i < n_units && !*abort; ++i) {
        const bool first = kk == 0, last = kk == nk - 1;
        const int buf = seg & 1;
        if (first) {
          if (!mbar_wait(&hdr->tmem_empty[buf], ((seg >> 1) & 1) ^ 1, abort, a.status)) break;
          tc_fence_after();
        }
        if (!mbar_wait(&hdr->full[s], ph, abort, a.status)) break;
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + static_cast<size_t>(s) * Lay::kStageBytes);
        const uint64_t ad = sw128_desc(sa), bd = sw128_desc(sa + kABytes);
#pragma unroll
        for (int k = 0; k < kBK / 32; ++k)
          mma_i8(tmem + buf * NT, ad + 2 * k, bd + 2 * k, idesc, (first && k == 0) ? 0u : 1u);
        mma_commit(&hdr->empty[s]);
        if (last) {
          mma_commit(&hdr->tmem_full[buf]);
          ++seg;
        }
        kk = last ? 0 : kk + 1;
        if (++s == S) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
  } else {
    // --------------------------------------------------------------- epilogue ----
    float *xs_s = hdr->xs;
    const int quad = warp & 3;               // TMEM lane quadrant this warp may access
    const int row = quad * 32 + lane;        // weight row within the tile
    const int et = threadIdx.x - 64;         // 0..255
    constexpr int kHalf = NT >= 32 ? NT / 2 : NT;
    const int cbeg = (et >> 7) * kHalf;      // this warp's token columns [cbeg, cbeg + kHalf)
    const bool drains = cbeg < NT;
    griddep_wait();  // activation scales, and the output buffer, belong to earlier kernels
    for (int t = et; t < NT; t += kEpi) {
      const int m = a.m0 + t;
      xs_s[t] = (a.out_kind == 0 && m < a.M) ? a.xs[m] : 0.0f;
    }
    epi_bar_sync(kEpi);
    for (int seg = 0; seg < my_tiles; ++seg) {
      const int tile = cid + seg * a.nclusters;
      const int buf = seg & 1;
      if (et < kBM) {  // this tile's weight scales, loaded while its K range still streams
        const int n = tile * kBM + et;
        hdr->wsc[buf][et] = (n < a.N && a.out_kind == 0) ? a.ws[n] : 0.0f;
      }
      // One thread waits (bounded); the named barrier then releases the others together, so
      // on a timeout all epilogue threads leave the loop at the same point.
      if (et == 0) {
        mbar_wait(&hdr->tmem_full[buf], (seg >> 1) & 1, abort, a.status);
        if (clustered && seg >= 1) {
          // the peers reduced the previous tile (receive buffers free) and this CTA's own
          // copies out of the staging tile have been read
          mbar_wait_cluster(&hdr->done, (seg - 1) & 1, abort, a.status);
          asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        }
      }
      epi_bar_sync(kEpi);
      if (*abort) break;
      tc_fence_after();
      if (a.out_kind == 2) {  // this CTA's int32 partial tile -> partial slice crank
        const int n = tile * kBM + row;
        int32_t *yp = static_cast<int32_t *>(a.y) + static_cast<size_t>(crank) * a.M * a.N;
        if (drains) {
#pragma unroll 1
          for (int c0 = cbeg; c0 < cbeg + kHalf; c0 += 16) {
            uint32_t v[16];
            tmem_ld16(tmem + (static_cast<uint32_t>(quad * 32) << 16) + buf * NT + c0, v);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int m = a.m0 + c0 + j;
              if (m < a.M && n < a.N) yp[static_cast<size_t>(m) * a.N + n] = static_cast<int32_t>(v[j]);
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&hdr->tmem_empty[buf]);
        continue;
      }
      if (C == 1) {
        const int n = tile * kBM + row;
        const float wsn = hdr->wsc[buf][row];
        if (drains) {
#pragma unroll 1
          for (int c0 = cbeg; c0 < cbeg + kHalf; c0 += 16) {
            uint32_t v[16];
            tmem_ld16(tmem + (static_cast<uint32_t>(quad * 32) << 16) + buf * NT + c0, v);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int t = c0 + j, m = a.m0 + t;
              if (m >= a.M || n >= a.N) continue;
              const int32_t accv = static_cast<int32_t>(v[j]);
              const size_t o = static_cast<size_t>(m) * a.N + n;
              if (a.out_kind == 1)
                static_cast<int32_t *>(a.y)[o] = accv;
              else
                static_cast<T *>(a.y)[o] =
                    from_f32<T>(__fmul_rn(__fmul_rn(static_cast<float>(accv), xs_s[t]), wsn));
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&hdr->tmem_empty[buf]);
        continue;
      }
      // ---- split-K: TMEM rows -> staging tile; one bulk copy per peer moves the peer's rows
      // into its receive buffer (completing on its barrier); then reduce the received rows ----
      if (drains) {
#pragma unroll 1
        for (int c0 = cbeg; c0 < cbeg + kHalf; c0 += 16) {
          uint32_t v[16];
          tmem_ld16(tmem + (static_cast<uint32_t>(quad * 32) << 16) + buf * NT + c0, v);
          tmem_wait_ld();
          int4 *dst = reinterpret_cast<int4 *>(part + row * Lay::kPartPitch + c0 * 4);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            dst[j] = make_int4(static_cast<int>(v[4 * j]), static_cast<int>(v[4 * j + 1]),
                               static_cast<int>(v[4 * j + 2]), static_cast<int>(v[4 * j + 3]));
        }
      }
      tc_fence_before();
      mbar_arrive(&hdr->tmem_empty[buf]);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      epi_bar_sync(kEpi);
      if (et == 0) {
        for (int q = 0; q < C; ++q) {
          const int q0 = (q * kBM + C - 1) / C, q1 = ((q + 1) * kBM + C - 1) / C;
          const uint32_t dst =
              mapa(smem_u32(recvb + static_cast<int>(crank) * slot_rows * Lay::kPartPitch), q);
          asm volatile(
              "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                  dst),
              "r"(smem_u32(part + q0 * Lay::kPartPitch)), "r"((q1 - q0) * Lay::kPartPitch),
              "r"(mapa(smem_u32(&hdr->recv), q))
              : "memory");
        }
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        mbar_wait_cluster(&hdr->recv, seg & 1, abort, a.status);
      }
      epi_bar_sync(kEpi);
      if (*abort) break;
      const int R = r1 - r0;
      const uint8_t *pb = recvb;
      const int items = R * (NT / 4);
      for (int idx = et; idx < items; idx += kEpi) {
        const int rl = idx % R, tq = idx / R;
        int4 acc = *reinterpret_cast<const int4 *>(pb + rl * Lay::kPartPitch + tq * 16);
        for (int q = 1; q < C; ++q) {
          const int4 v = *reinterpret_cast<const int4 *>(pb + (q * slot_rows + rl) * Lay::kPartPitch + tq * 16);
          acc.x += v.x;
          acc.y += v.y;
          acc.z += v.z;
          acc.w += v.w;
        }
        const int rr = r0 + rl, n = tile * kBM + rr;
        if (n >= a.N) continue;
        const int accs[4] = {acc.x, acc.y, acc.z, acc.w};
        const float wsn = hdr->wsc[buf][rr];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int t = 4 * tq + j, m = a.m0 + t;
          if (m >= a.M) continue;
          const size_t o = static_cast<size_t>(m) * a.N + n;
          if (a.out_kind == 1)
            static_cast<int32_t *>(a.y)[o] = accs[j];
          else
            static_cast<T *>(a.y)[o] =
                from_f32<T>(__fmul_rn(__fmul_rn(static_cast<float>(accs[j]), xs_s[t]), wsn));
        }
      }
      epi_bar_sync(kEpi);
      if (et == 0) {  // re-arm the receive buffer for the next tile, then let the senders in
        if (seg + 1 < my_tiles) mbar_expect_tx(&hdr->recv, recv_bytes);
        for (int q = 0; q < C; ++q) mbar_arrive_remote(&hdr->done, q);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (clustered) {  // no CTA leaves while a peer may still read its buffers or arrive on them
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
  }
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(Lay::kTmemCols)
                 : "memory");
}

// ----------------------------------------------------------------------- host side ----
int make_map(CUtensorMap *map, const void *base, int inner, int outer, int box_outer) {
  return make_map_2d(map, base, static_cast<uint64_t>(inner), static_cast<uint64_t>(outer),
                     static_cast<uint64_t>(inner), kBK, static_cast<uint32_t>(box_outer));
}

inline int pick_nt(int m) {
  return m <= 16 ? 16 : m <= 32 ? 32 : m <= 64 ? 64 : m <= 128 ? 128 : 256;
}

// Clusters of C CTAs that can be resident at once for this kernel (cached per device).
template <typename T, int NT>
int active_clusters(int C) {
  static std::mutex mu;
  static std::map<std::pair<int, int>, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  const auto key = std::make_pair(dev, C);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  using Lay = TcLayout<NT>;
  auto kern = gemm_tc_kernel<T, NT>;
  ensure_smem(reinterpret_cast<const void *>(kern), Lay::kSmem);
  int n = 0;
  if (C == 1) {
    n = sm_count();
  } else {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(C * (sm_count() / C), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = Lay::kSmem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = C;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
  }
  cache[key] = n;
  return n;
}

// Cluster size for a GEMM of n_tiles 128-row tiles x kc K chunks: the fewest chunk-times per
// CTA, counting each split tile's cluster reduction as about two chunks.
template <typename T, int NT>
int pick_split(int n_tiles, int kc, int *nclusters) {
  int best_c = 1, best_ncl = active_clusters<T, NT>(1);
  long best = static_cast<long>((n_tiles + best_ncl - 1) / best_ncl) * kc;
  if (NT <= 64) {
    for (int C = 2; C <= 8 && C <= kc; ++C) {
      const int ncl = active_clusters<T, NT>(C);
      if (ncl <= 0) continue;
      const long rounds = (n_tiles + ncl - 1) / ncl;
      const long cost = rounds * ((kc + C - 1) / C + 2);
      if (cost < best) {
        best = cost;
        best_c = C;
        best_ncl = ncl;
      }
    }
  }
  *nclusters = best_ncl < n_tiles ? best_ncl : n_tiles;
  return best_c;
}

// Split count for the partial-output mode (out_kind 2): CTA groups need no co-scheduling, so
// C CTAs of a group are any C of the one-per-SM CTAs. Fewest chunk-times per CTA; ties go to
// the smaller C (fewer partial bytes for the consumer to read).
inline int pick_split_partials(int n_tiles, int kc, int *ngroups) {
  const int sms = sm_count();
  int best_c = 1, best_g = sms < n_tiles ? sms : n_tiles;
  long best = static_cast<long>((n_tiles + sms - 1) / sms) * kc;
  for (int C = 2; C <= 8 && C <= kc; ++C) {
    const int g = sms / C;
    const long cost = static_cast<long>((n_tiles + g - 1) / g) * ((kc + C - 1) / C);
    if (cost < best) {
      best = cost;
      best_c = C;
      best_g = g < n_tiles ? g : n_tiles;
    }
  }
  *ngroups = best_g;
  return best_c;
}

template <typename T, int NT, bool PARTS>
int launch_tc_nt_impl(const CUtensorMap &mw, const CUtensorMap &mx, TcArgs args,
                      cudaStream_t st) {
  using Lay = TcLayout<NT, PARTS>;
  auto kern = gemm_tc_kernel<T, NT, PARTS>;
  ensure_smem(reinterpret_cast<const void *>(kern), Lay::kSmem);
  int ncl = 0;
  const int C = args.out_kind == 2 ? pick_split_partials(args.n_tiles, args.kc, &ncl)
                                   : pick_split<T, NT>(args.n_tiles, args.kc, &ncl);
  args.csplit = C;
  args.nclusters = ncl;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(C * ncl, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = Lay::kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = args.out_kind == 2 ? 1 : C;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, mw, mx, args);
  if (e != cudaSuccess) {
    record_cuda_error(e);
    return S8B_ERR_CUDA;
  }
  return check_launch();
}

template <typename T, int NT>
int launch_tc_nt(const CUtensorMap &mw, const CUtensorMap &mx, TcArgs args, cudaStream_t st) {
  return args.out_kind == 2 ? launch_tc_nt_impl<T, NT, false>(mw, mx, args, st)
                            : launch_tc_nt_impl<T, NT, true>(mw, mx, args, st);
}

template <typename T>
int launch_tc(const int8_t *xq, const float *xs, const int8_t *w, const float *ws, void *y,
              int out_kind, int M, int N, int K, void *workspace, cudaStream_t st,
              bool packed = false) {
  TcArgs args;
  args.xs = xs;
  args.ws = ws;
  args.y = y;
  args.status = static_cast<int32_t *>(workspace);
  args.out_kind = out_kind;
  args.M = M;
  args.N = N;
  args.K = K;
  args.n_tiles = (N + kBM - 1) / kBM;
  args.kc = K / kBK;
  args.wpacked = packed ? w : nullptr;
  CUtensorMap mw;
  int rc = S8B_OK;
  if (packed)
    memset(&mw, 0, sizeof(mw));
  else
    rc = make_map(&mw, w, K, N, kBM);
  if (rc) return rc;
  for (int m0 = 0; m0 < M; m0 += 256) {
    const int mt = M - m0 < 256 ? M - m0 : 256;
    const int nt = pick_nt(mt);
    CUtensorMap mx;
    rc = make_map(&mx, xq, K, M, nt);
    if (rc) return rc;
    args.m0 = m0;
    switch (nt) {
      case 16: rc = launch_tc_nt<T, 16>(mw, mx, args, st); break;
      case 32: rc = launch_tc_nt<T, 32>(mw, mx, args, st); break;
      case 64: rc = launch_tc_nt<T, 64>(mw, mx, args, st); break;
      case 128: rc = launch_tc_nt<T, 128>(mw, mx, args, st); break;
      default: rc = launch_tc_nt<T, 256>(mw, mx, args, st); break;
    }
    if (rc) return rc;
  }
  return S8B_OK;
}

}  // namespace
}  // namespace s8b

using namespace s8b;

extern "C" size_t s8b_gemm_tc_workspace_size(int M, int N) {
  (void)M;
  (void)N;
  return 256;  // the status word (split-K partials are reduced on chip)
}

extern "C" int s8b_gemm_w8a8_tc(const int8_t *xq, const float *xs, const int8_t *w,
                                const float *ws, void *y, int out_kind, int M, int N, int K,
                                int dtype, void *workspace, size_t workspace_bytes, void *stream) {
  if (!xq || !w || !y || (out_kind == 0 && (!xs || !ws))) return S8B_ERR_ARG;
  if (out_kind < 0 || out_kind > 2) return S8B_ERR_ARG;
  if (M < 0 || N <= 0 || K <= 0 || K % kBK != 0) return S8B_ERR_SHAPE;
  if (!aligned(xq, 16) || !aligned(w, 16)) return S8B_ERR_ALIGN;
  if (!workspace || workspace_bytes < s8b_gemm_tc_workspace_size(M, N)) return S8B_ERR_WORKSPACE;
  if (!aligned(workspace, 256)) return S8B_ERR_ALIGN;
  if (M == 0) return S8B_OK;
  S8B_DISPATCH_DTYPE(dtype, T,
                     return launch_tc<T>(xq, xs, w, ws, y, out_kind, M, N, K, workspace,
                                         (cudaStream_t)stream));
}

extern "C" int s8b_gemm_tc_split_count(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0 || K % kBK != 0) return S8B_ERR_SHAPE;
  int groups = 0;
  return pick_split_partials((N + kBM - 1) / kBM, K / kBK, &groups);
}

extern "C" size_t s8b_tc_packed_bytes(int N, int K) {
  if (N <= 0 || K <= 0 || K % kBK != 0) return 0;
  return static_cast<size_t>((N + kBM - 1) / kBM) * (K / kBK) * kABytes;
}

extern "C" int s8b_pack_weights_tc(const int8_t *w, int N, int K, int8_t *packed, void *stream) {
  if (!w || !packed) return S8B_ERR_ARG;
  if (N <= 0 || K <= 0 || K % kBK != 0) return S8B_ERR_SHAPE;
  if (!aligned(w, 16) || !aligned(packed, 16)) return S8B_ERR_ALIGN;
  pack_tc_kernel<<<4 * sm_count(), 256, 0, (cudaStream_t)stream>>>(w, N, K, packed);
  return check_launch();
}

extern "C" int s8b_gemm_w8a8_tc_packed(const int8_t *xq, const float *xs, const int8_t *wpacked,
                                       const float *ws, void *y, int out_kind, int M, int N,
                                       int K, int dtype, void *workspace,
                                       size_t workspace_bytes, void *stream) {
  if (!xq || !wpacked || !y || (out_kind == 0 && (!xs || !ws))) return S8B_ERR_ARG;
  if (out_kind < 0 || out_kind > 2) return S8B_ERR_ARG;
  if (M < 0 || N <= 0 || K <= 0 || K % kBK != 0) return S8B_ERR_SHAPE;
  if (!aligned(xq, 16) || !aligned(wpacked, 16)) return S8B_ERR_ALIGN;
  if (!workspace || workspace_bytes < s8b_gemm_tc_workspace_size(M, N)) return S8B_ERR_WORKSPACE;
  if (!aligned(workspace, 256)) return S8B_ERR_ALIGN;
  if (M == 0) return S8B_OK;
  S8B_DISPATCH_DTYPE(dtype, T,
                     return launch_tc<T>(xq, xs, wpacked, ws, y, out_kind, M, N, K, workspace,
                                         (cudaStream_t)stream, true));
}
