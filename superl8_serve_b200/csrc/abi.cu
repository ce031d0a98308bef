// Status plumbing of the C ABI.
#include <atomic>
#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"

namespace s8b {

static std::atomic<int> g_last_cuda_error{0};
static std::atomic<unsigned long long> g_launches{0};

void record_cuda_error(cudaError_t e) { g_last_cuda_error.store(static_cast<int>(e)); }

int check_launch(int launches) {
  g_launches.fetch_add(static_cast<unsigned long long>(launches));
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    record_cuda_error(e);
    return S8B_ERR_CUDA;
  }
  return S8B_OK;
}

static std::mutex g_smem_mu;
static std::map<std::pair<const void *, int>, size_t> g_smem_set;

void ensure_smem(const void *kernel, size_t bytes) {
  // Static shared memory counts against the same limit, so raise it for any dynamic size
  // beyond a few KB rather than only above 48 KB.
  if (bytes <= 8 * 1024) return;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_smem_mu);
  size_t &cur = g_smem_set[{kernel, dev}];
  if (cur >= bytes) return;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(bytes)) == cudaSuccess)
    cur = bytes;
}

}  // namespace s8b

extern "C" const char *s8b_strerror(int code) {
  switch (code) {
    case S8B_OK: return "ok";
    case S8B_ERR_SHAPE: return "unsupported or inconsistent sizes";
    case S8B_ERR_DTYPE: return "unsupported dtype or codec scheme";
    case S8B_ERR_ALIGN: return "pointer or leading dimension misaligned";
    case S8B_ERR_CUDA: return "CUDA runtime error (see s8b_last_cuda_error)";
    case S8B_ERR_PEER: return "peer memory not registered or peer access unavailable";
    case S8B_ERR_TIMEOUT: return "bounded device-side wait timed out";
    case S8B_ERR_WORKSPACE: return "workspace missing or too small";
    case S8B_ERR_ARG: return "null pointer or invalid argument";
    case S8B_ERR_SCRATCH_LIMIT:
      return "problem needs more scratch than the 16 MiB static limit of the no-allocation entry point";
    default: return "unknown s8b status";
  }
}

extern "C" int s8b_version(void) { return 1; }

extern "C" int s8b_last_cuda_error(void) { return s8b::g_last_cuda_error.load(); }

extern "C" unsigned long long s8b_launch_count(void) { return s8b::g_launches.load(); }
