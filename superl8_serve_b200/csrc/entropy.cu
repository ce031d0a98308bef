// Static byte-level rANS on the GPU: the wire format of the reference's optional entropy
// stage (superl8serve/dist/entropy.py: 32-bit state in [2^23, 2^31), frequencies normalised
// to M = 2^12, symbols coded in reverse, renormalisation bytes emitted low byte first, the
// final state flushed as 4 bytes low byte first; decode reads from the end).
//
// One rANS stream is a sequential chain (each symbol's state depends on the previous one),
// so a stream is one thread. A payload is cut into `n_streams` equal chunks, chunk i coded as
// an independent stream by thread i: with n_streams == 1 the output is byte for byte the
// reference's stream; more streams give parallelism (one thread each), and the caller keeps
// the per-stream lengths. Stream i owns the output region starting at 2*lo_i + 4*i
// (lo_i = i*n/n_streams), which bounds its size: the state stays below 2^31 and a symbol
// never emits more than 2 bytes (x_max >= 2^19), plus the 4 flush bytes.
#include "common.cuh"

namespace s8b {
namespace {

constexpr int kScaleBits = 12;
constexpr uint32_t kM = 1u << kScaleBits;
constexpr uint32_t kL = 1u << 23;
constexpr uint32_t kXMaxFactor = (kL >> kScaleBits) << 8;  // x_max(s) = factor * freq(s)
constexpr uint64_t kBadStream = ~0ull;

__host__ __device__ inline size_t stream_lo(size_t n, int S, int i) {
  return n * static_cast<size_t>(i) / static_cast<size_t>(S);
}
__host__ __device__ inline size_t stream_off(size_t n, int S, int i) {
  return 2 * stream_lo(n, S, i) + 4 * static_cast<size_t>(i);
}

__global__ void __launch_bounds__(256)
    rans_histogram_kernel(const uint8_t *__restrict__ sym, size_t n, uint32_t *counts) {
  __shared__ uint32_t h[256];
  h[threadIdx.x] = 0;
  __syncthreads();
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    atomicAdd(&h[sym[i]], 1u);
  __syncthreads();
  if (h[threadIdx.x]) atomicAdd(&counts[threadIdx.x], h[threadIdx.x]);
}

// Thread i encodes chunk i. A symbol whose frequency is 0 cannot be coded: the stream stops
// and reports kBadStream as its length.
__global__ void __launch_bounds__(128)
    rans_encode_kernel(const uint8_t *__restrict__ sym, size_t n, const int32_t *__restrict__ freqs,
                       int S, uint8_t *__restrict__ out, uint64_t *__restrict__ stream_len) {
  __shared__ uint32_t f_s[256], c_s[256];
  if (threadIdx.x == 0) {
    uint32_t c = 0;
    for (int s = 0; s < 256; ++s) {
      f_s[s] = static_cast<uint32_t>(freqs[s]);
      c_s[s] = c;
      c += f_s[s];
    }
  }
  __syncthreads();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= S) return;
  const size_t lo = stream_lo(n, S, i), hi = stream_lo(n, S, i + 1);
  uint8_t *o = out + stream_off(n, S, i);
  uint32_t state = kL;
  size_t pos = 0;
  for (size_t j = hi; j > lo; --j) {
    const uint32_t s = sym[j - 1];
    const uint32_t f = f_s[s];
    if (f == 0) {
      stream_len[i] = kBadStream;
      return;
    }
    const uint32_t x_max = kXMaxFactor * f;
    while (state >= x_max) {
      o[pos++] = static_cast<uint8_t>(state & 0xffu);
      state >>= 8;
    }
    state = ((state / f) << kScaleBits) + (state % f) + c_s[s];
  }
  for (int b = 0; b < 4; ++b) {
    o[pos++] = static_cast<uint8_t>(state & 0xffu);
    state >>= 8;
  }
  stream_len[i] = pos;
}

// Thread i decodes chunk i from its region (stream_len[i] bytes). Every read stays inside
// the stream's bytes; a stream that runs out early (corrupt input) stops and marks
// `bad` (the decoded symbols of that chunk are then incomplete).
__global__ void __launch_bounds__(128)
    rans_decode_kernel(const uint8_t *__restrict__ enc, const uint64_t *__restrict__ stream_len,
                       int S, const int32_t *__restrict__ freqs, size_t n,
                       uint8_t *__restrict__ out, int32_t *bad) {
  __shared__ uint32_t f_s[256], c_s[256];
  __shared__ uint8_t slot_sym[kM];
  if (threadIdx.x == 0) {
    uint32_t c = 0;
    for (int s = 0; s < 256; ++s) {
      f_s[s] = static_cast<uint32_t>(freqs[s]);
      c_s[s] = c;
      c += f_s[s];
    }
  }
  __syncthreads();
  for (int s = 0; s < 256; ++s)
    for (uint32_t k = threadIdx.x; k < f_s[s]; k += blockDim.x)
      if (c_s[s] + k < kM) slot_sym[c_s[s] + k] = static_cast<uint8_t>(s);
  __syncthreads();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= S) return;
  const size_t lo = stream_lo(n, S, i), hi = stream_lo(n, S, i + 1);
  const uint8_t *b = enc + stream_off(n, S, i);
  const uint64_t len = stream_len[i];
  if (len < 4 || len > 2 * (hi - lo) + 4) {
    if (hi > lo) atomicExch(bad, 1);
    return;
  }
  size_t pos = len - 4;
  uint32_t state = static_cast<uint32_t>(b[pos]) | (static_cast<uint32_t>(b[pos + 1]) << 8) |
                   (static_cast<uint32_t>(b[pos + 2]) << 16) |
                   (static_cast<uint32_t>(b[pos + 3]) << 24);
  for (size_t j = lo; j < hi; ++j) {
    const uint32_t slot = state & (kM - 1);
    const uint32_t s = slot_sym[slot];
    state = f_s[s] * (state >> kScaleBits) + slot - c_s[s];
    while (state < kL) {
      if (pos == 0) {
        atomicExch(bad, 1);
        return;
      }
      state = (state << 8) | b[--pos];
    }
    out[j] = static_cast<uint8_t>(s);
  }
}

}  // namespace
}  // namespace s8b

using namespace s8b;

extern "C" size_t s8b_rans_encoded_capacity(size_t n, int n_streams) {
  if (n_streams < 1) return 0;
  return 2 * n + 4 * static_cast<size_t>(n_streams);
}

extern "C" size_t s8b_rans_stream_offset(size_t n, int n_streams, int i) {
  if (n_streams < 1 || i < 0 || i > n_streams) return 0;
  return stream_off(n, n_streams, i);
}

extern "C" int s8b_rans_histogram(const uint8_t *sym, size_t n, uint32_t *counts, void *stream) {
  if (!sym || !counts) return S8B_ERR_ARG;
  const cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(counts, 0, 256 * sizeof(uint32_t), st);
  if (e != cudaSuccess) {
    record_cuda_error(e);
    return S8B_ERR_CUDA;
  }
  if (n == 0) return S8B_OK;
  const size_t want = (n + 255) / 256;
  const unsigned blocks = static_cast<unsigned>(want < 2048 ? want : 2048);
  rans_histogram_kernel<<<blocks, 256, 0, st>>>(sym, n, counts);
  return check_launch();
}

extern "C" int s8b_rans_encode(const uint8_t *sym, size_t n, const int32_t *freqs, int n_streams,
                               uint8_t *out, size_t out_capacity, uint64_t *stream_len,
                               void *stream) {
  if (!sym || !freqs || !out || !stream_len) return S8B_ERR_ARG;
  if (n_streams < 1 || static_cast<size_t>(n_streams) > (n > 0 ? n : 1)) return S8B_ERR_SHAPE;
  if (out_capacity < s8b_rans_encoded_capacity(n, n_streams)) return S8B_ERR_WORKSPACE;
  const unsigned blocks = static_cast<unsigned>((n_streams + 127) / 128);
  rans_encode_kernel<<<blocks, 128, 0, (cudaStream_t)stream>>>(sym, n, freqs, n_streams, out,
                                                                stream_len);
  return check_launch();
}

extern "C" int s8b_rans_decode(const uint8_t *enc, const uint64_t *stream_len, int n_streams,
                               const int32_t *freqs, size_t n, uint8_t *out, int32_t *bad,
                               void *stream) {
  if (!enc || !stream_len || !freqs || !out || !bad) return S8B_ERR_ARG;
  if (n_streams < 1 || static_cast<size_t>(n_streams) > (n > 0 ? n : 1)) return S8B_ERR_SHAPE;
  const cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(bad, 0, sizeof(int32_t), st);
  if (e != cudaSuccess) {
    record_cuda_error(e);
    return S8B_ERR_CUDA;
  }
  const unsigned blocks = static_cast<unsigned>((n_streams + 127) / 128);
  rans_decode_kernel<<<blocks, 128, 0, st>>>(enc, stream_len, n_streams, freqs, n, out, bad);
  return check_launch();
}
