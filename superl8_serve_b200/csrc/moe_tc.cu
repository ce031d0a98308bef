// Grouped W8A8 expert GEMM of the sparse-MoE FFN on the 5th-generation tensor cores
// (tcgen05.mma kind::i8), and the row gather that feeds it.
//
// y[r, n] = bf16((f32(sum_k x[r, k] * w[e, n, k]) * xs[r]) * ws[e, n]) for every sorted
// assignment row r of expert e (rows offsets[e] .. offsets[e + 1] - 1). The sum is an exact
// int32, so the result is bit-identical to the CUDA-core grouped kernel (s8b_moe_gemm_grouped).
//
// The MMA is issued swap-AB as in the dense GEMM: A = 128 weight rows of one expert x 32
// K-bytes (the HBM stream fills the MMA's 128-row dimension), B = the expert's token rows
// (a handful per expert at decode batch sizes) x 32 K-bytes, D = 128 x N int32 in TMEM with N
// the expert's row count rounded up to 16 (at most 64 per pass). Work units are (expert,
// 128-row weight tile, pass of 64 token rows); a persistent grid walks them round-robin,
// passes outermost, so every CTA gets its share of first passes and the rare second passes
// (experts with more than 64 rows) come last. Weight tiles come straight from the [E * N, K]
// weight array by 2-D tensor copies (no packed copy); token rows come from the rows already
// gathered into assignment order (s8b_moe_gather_rows), so an expert's rows are contiguous
// and one 16-row tensor copy per 16 rows fetches them.
//
// Roles (320 threads): warp 0 issues the copies, warp 1 the MMAs (one thread) and owns the
// TMEM allocation, warps 2-9 drain TMEM (two warps per lane quadrant, each half of the token
// columns). The accumulator is double-buffered in TMEM. Every mbarrier wait is bounded.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "tcgen05.cuh"

namespace s8b {
namespace {

using namespace tc;

constexpr int kGM = 128;              // weight rows per tile (MMA M)
constexpr int kGK = 128;              // K bytes per stage
constexpr int kGA = kGM * kGK;        // 16 KB weight tile per stage
constexpr int kGNT = 64;              // token rows per pass (MMA N <= 64)
constexpr int kGRowBox = 16;          // token rows per tensor copy
constexpr int kGStage = kGA + kGNT * kGK;  // 24 KB
constexpr int kGStages = 8;
constexpr int kGThreads = 320;
constexpr int kGEpi = 256;
constexpr int kGMaxE = 512;           // experts per launch (their offsets sit in shared memory)
constexpr int kGTmemCols = 2 * kGNT;

struct GHdr {
  uint64_t full[kGStages];
  uint64_t empty[kGStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint32_t tmem_base;
  int abort;
  float xs[2][kGNT];  // the pass's token scales, per TMEM buffer
  int stop[2];        // epilogue: leave the loop (broadcast by one thread), per TMEM buffer
  int off[kGMaxE + 1];
};
constexpr size_t kGSmem = 1024 + static_cast<size_t>(kGStages) * kGStage + sizeof(GHdr);

struct GArgs {
  const float *xs;      // [A] token scales, assignment order
  const float *ws;      // [E, N] weight row scales
  const int32_t *offsets;  // [E + 1] assignment rows of each expert (absolute row numbers)
  void *y;              // [rows, N] outputs, assignment order
  int32_t *status;      // S8B_ERR_TIMEOUT on a bounded wait that gave up
  int N, K, E, tiles, passes;
};

// The walk over units shared by every role: v = pass * (E * tiles) + e * tiles + tile.
struct GUnit {
  int e, tile, row0, rows;  // rows: this pass's token rows (<= 64), 0 = empty unit
};
__device__ __forceinline__ GUnit g_unit(int v, const GArgs &a, const int *off) {
  const int et = a.E * a.tiles;
  const int pass = v / et, r = v - pass * et, e = r / a.tiles, tile = r - e * a.tiles;
  const int n = off[e + 1] - off[e] - pass * kGNT;
  return {e, tile, off[e] + pass * kGNT, n <= 0 ? 0 : (n < kGNT ? n : kGNT)};
}

template <typename T>
__global__ void __launch_bounds__(kGThreads, 1)
    moe_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_w,
                       const __grid_constant__ CUtensorMap tmap_x, GArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  GHdr *hdr = reinterpret_cast<GHdr *>(smem + static_cast<size_t>(kGStages) * kGStage);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  griddep_launch();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kGStages; ++s) {
      mbar_init(&hdr->full[s], 1);
      mbar_init(&hdr->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&hdr->tmem_full[b], 1);
      mbar_init(&hdr->tmem_empty[b], kGEpi);
    }
    hdr->abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&hdr->tmem_base)),
                 "r"(kGTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  griddep_wait();  // the routing (offsets) and the gathered rows come from earlier kernels
  for (int i = threadIdx.x; i <= a.E; i += kGThreads) hdr->off[i] = a.offsets[i];
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = hdr->tmem_base;
  volatile int *abort = &hdr->abort;
  const int V = a.passes * a.E * a.tiles;
  const int kc = a.K / kGK;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer ----
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_w)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_x)) : "memory");
      int s = 0;
      uint32_t ph = 0;  // phase parity of stage s's next fill
      long long issued = 0;
      bool ok = true;
      for (int v = blockIdx.x; v < V && ok; v += gridDim.x) {
        const GUnit u = g_unit(v, a, hdr->off);
        if (u.rows == 0) continue;
        const int nb = (u.rows + kGRowBox - 1) / kGRowBox;
        const uint32_t bytes = kGA + nb * kGRowBox * kGK;
        for (int kk = 0; kk < kc; ++kk) {
          if (issued >= kGStages && !mbar_wait(&hdr->empty[s], ph ^ 1, abort, a.status)) {
            ok = false;
            break;
          }
          uint8_t *st = smem + static_cast<size_t>(s) * kGStage;
          mbar_expect_tx(&hdr->full[s], bytes);
          tma_load_2d(st, &tmap_w, kk * kGK, u.e * a.N + u.tile * kGM, &hdr->full[s]);
          for (int i = 0; i < nb; ++i)
            tma_load_2d(st + kGA + i * kGRowBox * kGK, &tmap_x, kk * kGK, u.row0 + i * kGRowBox,
                        &hdr->full[s]);
          ++issued;
          if (++s == kGStages) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (*abort) {  // let the copies already issued land before shared memory goes away
        const long long first = issued > kGStages ? issued - kGStages : 0;
        for (long long i = first; i < issued; ++i)
          mbar_drain(&hdr->full[i % kGStages], static_cast<uint32_t>((i / kGStages) & 1));
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------- MMA issuer ----
    if (lane == 0) {
      int s = 0, seg = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int v = blockIdx.x; v < V && ok; v += gridDim.x) {
        const GUnit u = g_unit(v, a, hdr->off);
        if (u.rows == 0) continue;
        const int ncol = (u.rows + 15) & ~15;
        const uint32_t idesc = i8_idesc(kGM, ncol);
        const int buf = seg & 1;
        if (!mbar_wait(&hdr->tmem_empty[buf], ((seg >> 1) & 1) ^ 1, abort, a.status)) break;
        tc_fence_after();
        for (int kk = 0; kk < kc; ++kk) {
          if (!mbar_wait(&hdr->full[s], ph, abort, a.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + static_cast<size_t>(s) * kGStage);
          const uint64_t ad = sw128_desc(sa), bd = sw128_desc(sa + kGA);
#pragma unroll
          for (int k = 0; k < kGK / 32; ++k)
            mma_i8(tmem + buf * kGNT, ad + 2 * k, bd + 2 * k, idesc, (kk == 0 && k == 0) ? 0u : 1u);
          mma_commit(&hdr->empty[s]);
          if (++s == kGStages) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(&hdr->tmem_full[buf]);
        ++seg;
      }
    }
  } else {
    // --------------------------------------------------------------- epilogue ----
    const int quad = warp & 3;             // TMEM lane quadrant this warp may access
    const int row = quad * 32 + lane;      // weight row within the tile
    const int et = threadIdx.x - 64;       // 0..255
    const int cbeg = (et >> 7) * (kGNT / 2);  // this warp's token columns [cbeg, cbeg + 32)
    int seg = 0;
    for (int v = blockIdx.x; v < V; v += gridDim.x) {
      const GUnit u = g_unit(v, a, hdr->off);
      if (u.rows == 0) continue;
      const int buf = seg & 1;
      if (et < u.rows) hdr->xs[buf][et] = a.xs[u.row0 + et];
      // one thread waits (bounded) and decides for all, so every epilogue thread leaves the
      // loop at the same barrier
      if (et == 0)
        hdr->stop[buf] = !mbar_wait(&hdr->tmem_full[buf], (seg >> 1) & 1, abort, a.status) || *abort;
      epi_bar_sync(kGEpi);
      if (hdr->stop[buf]) break;
      tc_fence_after();
      const int n = u.tile * kGM + row;
      const float wsn = n < a.N ? a.ws[static_cast<size_t>(u.e) * a.N + n] : 0.0f;
      if (cbeg < u.rows) {
#pragma unroll
        for (int c0 = 0; c0 < kGNT / 2; c0 += 16) {
          uint32_t vals[16];
          tmem_ld16(tmem + (static_cast<uint32_t>(quad * 32) << 16) + buf * kGNT + cbeg + c0, vals);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int t = cbeg + c0 + j;
            if (t >= u.rows || n >= a.N) continue;
            const float y = __fmul_rn(__fmul_rn(static_cast<float>(static_cast<int32_t>(vals[j])),
                                                hdr->xs[buf][t]),
                                      wsn);
            static_cast<T *>(a.y)[static_cast<size_t>(u.row0 + t) * a.N + n] = from_f32<T>(y);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&hdr->tmem_empty[buf]);
      ++seg;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kGTmemCols)
                 : "memory");
}

// Row gather into assignment order: xg[r] = xq[index[r]], xgs[r] = xs[index[r]].
__global__ void __launch_bounds__(128)
    moe_gather_rows_kernel(const int8_t *__restrict__ xq, const float *__restrict__ xs,
                           const int32_t *__restrict__ index, int K, int8_t *__restrict__ xg,
                           float *__restrict__ xgs) {
  griddep_launch();
  griddep_wait();
  const int r = blockIdx.x, src = index[r];
  const int4 *s = reinterpret_cast<const int4 *>(xq + static_cast<size_t>(src) * K);
  int4 *d = reinterpret_cast<int4 *>(xg + static_cast<size_t>(r) * K);
  for (int i = threadIdx.x; i < K / 16; i += blockDim.x) d[i] = s[i];
  if (threadIdx.x == 0) xgs[r] = xs[src];
}

}  // namespace
}  // namespace s8b

using namespace s8b;

extern "C" int s8b_moe_gather_rows(const int8_t *xq, const float *xs, const int32_t *index, int A,
                                   int K, int8_t *xg, float *xgs, void *stream) {
  if (!xq || !xs || !index || !xg || !xgs) return S8B_ERR_ARG;
  if (A < 0 || K <= 0 || K % 16 != 0) return S8B_ERR_SHAPE;
  if (!aligned(xq, 16) || !aligned(xg, 16)) return S8B_ERR_ALIGN;
  if (A == 0) return S8B_OK;
  launch_pdl(moe_gather_rows_kernel, A, 128, 0, (cudaStream_t)stream, xq, xs, index, K, xg, xgs);
  return check_launch();
}

extern "C" int s8b_moe_gemm_grouped_tc(const int8_t *xg, const float *xgs, const int8_t *w,
                                       const float *ws, const int32_t *expert_offsets, void *y,
                                       int A, int N, int K, int E, int max_rows, int32_t *status,
                                       int dtype, void *stream) {
  if (!xg || !xgs || !w || !ws || !expert_offsets || !y || !status) return S8B_ERR_ARG;
  if (A < 0 || N <= 0 || K <= 0 || K % kGK != 0 || E <= 0 || E > kGMaxE || max_rows < 0)
    return S8B_ERR_SHAPE;
  if (!aligned(xg, 16) || !aligned(w, 16)) return S8B_ERR_ALIGN;
  if (A == 0 || max_rows == 0) return S8B_OK;
  CUtensorMap mw, mx;
  if (make_map_2d(&mw, w, static_cast<uint64_t>(K), static_cast<uint64_t>(E) * N,
                  static_cast<uint64_t>(K), kGK, kGM) ||
      make_map_2d(&mx, xg, static_cast<uint64_t>(K), static_cast<uint64_t>(A),
                  static_cast<uint64_t>(K), kGK, kGRowBox))
    return S8B_ERR_ALIGN;
  GArgs a;
  a.xs = xgs;
  a.ws = ws;
  a.offsets = expert_offsets;
  a.y = y;
  a.status = status;
  a.N = N;
  a.K = K;
  a.E = E;
  a.tiles = (N + kGM - 1) / kGM;
  a.passes = (max_rows + kGNT - 1) / kGNT;
  const long long V = static_cast<long long>(a.passes) * E * a.tiles;
  if (V > 0x7fffffffLL) return S8B_ERR_SHAPE;
  const int grid = static_cast<int>(V < sm_count() ? V : sm_count());
  S8B_DISPATCH_DTYPE(dtype, T, {
    auto kern = moe_gemm_tc_kernel<T>;
    ensure_smem(reinterpret_cast<const void *>(kern), kGSmem);
    launch_pdl(kern, grid, kGThreads, kGSmem, (cudaStream_t)stream, mw, mx, a);
    return check_launch();
  });
}
