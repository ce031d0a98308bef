// W8A8 GEMM on the 5th-generation tensor cores (tcgen05.mma kind::i8) for decode token counts
// that make the contraction dense enough (16..256 tokens per launch).
//
// Shape: y[m, n] = dequant( sum_k xq[m, k] * w[n, k] ). The MMA is issued "swap-AB":
// A = 128 weight rows x 32 K-bytes, B = NT tokens x 32 K-bytes, D = 128 x NT int32 in TMEM,
// so the weight matrix (the HBM stream) fills the 128-row MMA dimension and the small token
// count is the N dimension.
//
// Work split. A unit is one 128-row x 128-byte weight chunk (16 KB). The units of all row
// tiles are laid out tile-major and cut into one contiguous range per persistent CTA (one CTA
// per SM), so every SM streams the same number of weight bytes whatever N and K are. A range
// that covers a whole row tile stores the result directly; ranges that cover part of a tile
// add their int32 partial sums into a workspace with red.global.add (exact: integer addition
// is associative), and the CTA that completes a tile's K range (per-tile counter) dequantizes,
// stores, and clears the workspace tile and counter for the next launch.
//
// Roles (192 threads): warp 0 issues TMA loads (128B swizzle, CTA-local destination), warp 1 issues the
// MMAs (one thread) and owns the TMEM allocation, warps 2-5 drain TMEM (32 lanes each). The
// accumulator is double-buffered in TMEM so a tile's epilogue overlaps the next tile's MMAs.
// Every mbarrier wait is bounded: on timeout the kernel records S8B_ERR_TIMEOUT in the
// workspace status word, lets in-flight copies land, frees TMEM and returns.
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
constexpr int kThreads = 192;
constexpr int kMaxStages = 8;
constexpr int kSmemBudget = 220 * 1024;

struct TcSmemHeader {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint32_t tmem_base;
  int abort;
  int is_last;
  float xs[256];  // per-token activation scales of this launch's token tile
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

template <int NT>
struct TcLayout {
  static constexpr int kBBytes = NT * kBK;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages =
      (kSmemBudget - 3072) / kStageBytes < kMaxStages ? (kSmemBudget - 3072) / kStageBytes
                                                      : kMaxStages;
  static constexpr int kTmemCols = 2 * NT < 32 ? 32 : 2 * NT;
  static constexpr size_t kSmem = 1024 + static_cast<size_t>(kStages) * kStageBytes + 2048;
};

struct TcArgs {
  const int8_t *wpacked;  // weights pre-packed into shared-memory images (null: TMA 2D path)
  const float *xs;
  const float *ws;
  void *y;
  int32_t *acc;       // workspace [NT][N] int32 (zero between launches)
  int32_t *counters;  // workspace [n_tiles]
  int32_t *status;    // workspace status word
  int out_kind, M, N, K, m0, n_tiles, kc;
};

template <typename T, int NT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_w,
                   const __grid_constant__ CUtensorMap tmap_x, TcArgs a) {
  using Lay = TcLayout<NT>;
  constexpr int S = Lay::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  TcSmemHeader *hdr = reinterpret_cast<TcSmemHeader *>(smem + static_cast<size_t>(S) * Lay::kStageBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const long long U = static_cast<long long>(a.n_tiles) * a.kc;
  const long long u0 = U * blockIdx.x / gridDim.x;
  const long long u1 = U * (blockIdx.x + 1) / gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&hdr->full[s], 1);
      mbar_init(&hdr->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&hdr->tmem_full[b], 1);
      mbar_init(&hdr->tmem_empty[b], 128);
    }
    hdr->abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
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
  tc_fence_after();
  const uint32_t tmem = hdr->tmem_base;
  volatile int *abort = &hdr->abort;

  if (warp == 0) {
    // ------------------------------------------------------------- TMA producer ----
    if (lane == 0) {
      long long issued = 0;
      for (long long u = u0; u < u1; ++u, ++issued) {
        const int s = static_cast<int>(issued % S);
        const uint32_t ph = static_cast<uint32_t>((issued / S) & 1);
        if (!mbar_wait(&hdr->empty[s], ph ^ 1, abort, a.status)) break;
        uint8_t *sa = smem + static_cast<size_t>(s) * Lay::kStageBytes;
        const int tile = static_cast<int>(u / a.kc), kk = static_cast<int>(u % a.kc);
        mbar_expect_tx(&hdr->full[s], Lay::kStageBytes);
        if (a.wpacked)
          bulk_load(sa, a.wpacked + static_cast<size_t>(u) * kABytes, kABytes, &hdr->full[s]);
        else
          tma_load_2d(sa, &tmap_w, kk * kBK, tile * kBM, &hdr->full[s]);
        tma_load_2d(sa + kABytes, &tmap_x, kk * kBK, a.m0, &hdr->full[s]);
      }
      if (*abort) {
        // let the copies already issued land before the CTA's shared memory goes away
        const long long first = issued > S ? issued - S : 0;
        for (long long i = first; i < issued; ++i) {
          const uint64_t t0 = now_ns();
          while (!mbar_try_wait(&hdr->full[i % S], static_cast<uint32_t>((i / S) & 1)) &&
                 now_ns() - t0 < 100000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------- MMA issuer ----
    if (lane == 0) {
      constexpr uint32_t idesc = i8_idesc(kBM, NT);
      long long it = 0;
      int seg = 0;
      for (long long u = u0; u < u1 && !*abort; ++u, ++it) {
        const int kk = static_cast<int>(u % a.kc);
        const bool first = (u == u0) || kk == 0;
        const bool last = (u == u1 - 1) || kk == a.kc - 1;
        const int buf = seg & 1;
        if (first) {
          if (!mbar_wait(&hdr->tmem_empty[buf], ((seg >> 1) & 1) ^ 1, abort, a.status)) break;
          tc_fence_after();
        }
        const int s = static_cast<int>(it % S);
        if (!mbar_wait(&hdr->full[s], static_cast<uint32_t>((it / S) & 1), abort, a.status)) break;
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
      }
    }
  } else {
    // --------------------------------------------------------------- epilogue ----
    float *xs_s = hdr->xs;
    const int quad = warp & 3;              // TMEM lane quadrant this warp may access
    const int row = quad * 32 + lane;       // weight row within the tile
    const int et = threadIdx.x - 64;        // 0..127
    for (int t = et; t < NT; t += 128) {
      const int m = a.m0 + t;
      xs_s[t] = (a.out_kind == 0 && m < a.M) ? a.xs[m] : 0.0f;
    }
    epi_bar_sync();
    int seg = 0;
    long long u = u0;
    while (u < u1) {
      const int tile = static_cast<int>(u / a.kc);
      const int kk0 = static_cast<int>(u % a.kc);
      const long long tile_end = static_cast<long long>(tile + 1) * a.kc;
      const long long ue = u1 < tile_end ? u1 : tile_end;
      const int nk = static_cast<int>(ue - u);
      const bool whole = kk0 == 0 && nk == a.kc;
      const int buf = seg & 1;
      // One thread waits (bounded); the named barrier then releases the other 127 together,
      // so on a timeout all epilogue threads leave the loop at the same point.
      if (et == 0) mbar_wait(&hdr->tmem_full[buf], (seg >> 1) & 1, abort, a.status);
      epi_bar_sync();
      if (*abort) break;
      tc_fence_after();
      const int n = tile * kBM + row;
      const float wsn = (n < a.N && a.out_kind == 0) ? a.ws[n] : 0.0f;
#pragma unroll 1
      for (int c0 = 0; c0 < NT; c0 += 16) {
        uint32_t v[16];
        tmem_ld16(tmem + (static_cast<uint32_t>(quad * 32) << 16) + buf * NT + c0, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int t = c0 + j, m = a.m0 + t;
          if (m >= a.M || n >= a.N) continue;
          const int32_t accv = static_cast<int32_t>(v[j]);
          if (whole) {
            const size_t o = static_cast<size_t>(m) * a.N + n;
            if (a.out_kind == 1)
              static_cast<int32_t *>(a.y)[o] = accv;
            else
              static_cast<T *>(a.y)[o] =
                  from_f32<T>(__fmul_rn(__fmul_rn(static_cast<float>(accv), xs_s[t]), wsn));
          } else {
            atomicAdd(a.acc + static_cast<size_t>(t) * a.N + n, accv);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&hdr->tmem_empty[buf]);
      if (!whole) {
        __threadfence();
        epi_bar_sync();
        if (et == 0) {
          const int old = atomicAdd(a.counters + tile, nk);
          hdr->is_last = (old + nk == a.kc);
        }
        epi_bar_sync();
        if (hdr->is_last) {
          __threadfence();
          // 16 independent L2 loads in flight per thread, then the stores (a load/store loop
          // would serialise one L2 round trip per token on possible aliasing).
#pragma unroll 1
          for (int t0 = 0; t0 < NT; t0 += 16) {
            int32_t vals[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int m = a.m0 + t0 + j;
              vals[j] = (m < a.M && n < a.N)
                            ? __ldcg(a.acc + static_cast<size_t>(t0 + j) * a.N + n) : 0;
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int m = a.m0 + t0 + j;
              if (m >= a.M || n >= a.N) continue;
              a.acc[static_cast<size_t>(t0 + j) * a.N + n] = 0;
              const size_t o = static_cast<size_t>(m) * a.N + n;
              if (a.out_kind == 1)
                static_cast<int32_t *>(a.y)[o] = vals[j];
              else
                static_cast<T *>(a.y)[o] = from_f32<T>(
                    __fmul_rn(__fmul_rn(static_cast<float>(vals[j]), xs_s[t0 + j]), wsn));
            }
          }
          if (et == 0) a.counters[tile] = 0;
        }
        epi_bar_sync();
      }
      ++seg;
      u = ue;
    }
  }
  tc_fence_before();
  __syncthreads();
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

size_t ws_layout(int M, int N, size_t *counters_off, size_t *acc_off) {
  const int nt = pick_nt(M < 256 ? M : 256);
  const size_t n_tiles = (static_cast<size_t>(N) + kBM - 1) / kBM;
  *counters_off = 256;
  *acc_off = (256 + n_tiles * 4 + 255) / 256 * 256;
  return *acc_off + static_cast<size_t>(nt) * N * 4;
}

template <typename T, int NT>
int launch_tc_nt(const CUtensorMap &mw, const CUtensorMap &mx, const TcArgs &args, cudaStream_t st) {
  using Lay = TcLayout<NT>;
  auto kern = gemm_tc_kernel<T, NT>;
  ensure_smem(reinterpret_cast<const void *>(kern), Lay::kSmem);
  const long long U = static_cast<long long>(args.n_tiles) * args.kc;
  const int grid = static_cast<int>(U < sm_count() ? U : sm_count());
  kern<<<grid, kThreads, Lay::kSmem, st>>>(mw, mx, args);
  return check_launch();
}

template <typename T>
int launch_tc(const int8_t *xq, const float *xs, const int8_t *w, const float *ws, void *y,
              int out_kind, int M, int N, int K, void *workspace, cudaStream_t st,
              bool packed = false) {
  size_t coff, aoff;
  ws_layout(M, N, &coff, &aoff);
  uint8_t *wsb = static_cast<uint8_t *>(workspace);
  TcArgs args;
  args.xs = xs;
  args.ws = ws;
  args.y = y;
  args.status = reinterpret_cast<int32_t *>(wsb);
  args.counters = reinterpret_cast<int32_t *>(wsb + coff);
  args.acc = reinterpret_cast<int32_t *>(wsb + aoff);
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
  size_t c, a;
  return ws_layout(M, N, &c, &a);
}

extern "C" int s8b_gemm_w8a8_tc(const int8_t *xq, const float *xs, const int8_t *w,
                                const float *ws, void *y, int out_kind, int M, int N, int K,
                                int dtype, void *workspace, size_t workspace_bytes, void *stream) {
  if (!xq || !w || !y || (out_kind == 0 && (!xs || !ws))) return S8B_ERR_ARG;
  if (out_kind != 0 && out_kind != 1) return S8B_ERR_ARG;
  if (M < 0 || N <= 0 || K <= 0 || K % kBK != 0) return S8B_ERR_SHAPE;
  if (!aligned(xq, 16) || !aligned(w, 16)) return S8B_ERR_ALIGN;
  if (!workspace || workspace_bytes < s8b_gemm_tc_workspace_size(M, N)) return S8B_ERR_WORKSPACE;
  if (!aligned(workspace, 256)) return S8B_ERR_ALIGN;
  if (M == 0) return S8B_OK;
  S8B_DISPATCH_DTYPE(dtype, T,
                     return launch_tc<T>(xq, xs, w, ws, y, out_kind, M, N, K, workspace,
                                         (cudaStream_t)stream));
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
  if (out_kind != 0 && out_kind != 1) return S8B_ERR_ARG;
  if (M < 0 || N <= 0 || K <= 0 || K % kBK != 0) return S8B_ERR_SHAPE;
  if (!aligned(xq, 16) || !aligned(wpacked, 16)) return S8B_ERR_ALIGN;
  if (!workspace || workspace_bytes < s8b_gemm_tc_workspace_size(M, N)) return S8B_ERR_WORKSPACE;
  if (!aligned(workspace, 256)) return S8B_ERR_ALIGN;
  if (M == 0) return S8B_OK;
  S8B_DISPATCH_DTYPE(dtype, T,
                     return launch_tc<T>(xq, xs, wpacked, ws, y, out_kind, M, N, K, workspace,
                                         (cudaStream_t)stream, true));
}
