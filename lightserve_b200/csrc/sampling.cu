// Greedy next-token selection for the decode step.
//
// Replaces lightserve's `logits[:, -1, :].argmax(dim=-1)` followed by the
// write of the next id (model/cuda_graph_decode.py:114-118; torch.argmax:
// the first index of the maximum, a NaN counts as the maximum) and, for the
// paged decode runner, the position increment of every sequence -- one
// launch instead of three torch kernels. One 1024-thread CTA per row; 16-byte
// loads when the row is aligned.
#include "common.cuh"

namespace lsb {

// (value, index) order of torch.argmax: NaN first, then larger values, then
// the smaller index.
__device__ __forceinline__ bool argmax_better(float a, int ia, float b, int ib) {
  const bool na = a != a, nb = b != b;
  if (na != nb) return na;
  if (!na && a != b) return a > b;
  return ia < ib;
}

template <typename T>
__global__ void __launch_bounds__(1024)
greedy_next_kernel(const T* __restrict__ logits, int64_t ld, int V, int64_t* __restrict__ tokens,
                   int64_t* __restrict__ positions) {
  allow_dependents();
  wait_prerequisites();
  const T* row = logits + (int64_t)blockIdx.x * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  constexpr int VEC = 16 / sizeof(T);
  const bool vec = (reinterpret_cast<uintptr_t>(row) & 15) == 0;
  const int nv = vec ? V / VEC : 0;
  // Four 16-byte loads in flight per thread before any is consumed: one
  // row is only ~64 KiB, so the time is load latency, not bandwidth.
  constexpr int U = 4;
  for (int c0 = threadIdx.x; c0 < nv; c0 += U * blockDim.x) {
    Vec16<T> v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + u * blockDim.x;
      if (c < nv) v[u] = ld_vec16_stream(row + c * VEC);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + u * blockDim.x;
      if (c < nv) {
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          const float f = to_f(v[u].v[j]);
          if (argmax_better(f, c * VEC + j, best, bi)) { best = f; bi = c * VEC + j; }
        }
      }
    }
  }
  for (int i = nv * VEC + threadIdx.x; i < V; i += blockDim.x) {
    const float f = to_f(row[i]);
    if (argmax_better(f, i, best, bi)) { best = f; bi = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (argmax_better(ob, oi, best, bi)) { best = ob; bi = oi; }
  }
  __shared__ float sb[32];
  __shared__ int si[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sb[warp] = best; si[warp] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (argmax_better(sb[w], si[w], best, bi)) { best = sb[w]; bi = si[w]; }
    tokens[blockIdx.x] = bi;
    if (positions != nullptr) positions[blockIdx.x] += 1;
  }
}

}  // namespace lsb

extern "C" int lsb_greedy_next(const void* logits, int64_t S, int64_t V, int64_t ld, int dtype,
                               int64_t* tokens, int64_t* positions, void* stream) {
  LSB_CHECK_ARG(S >= 0 && V > 0 && ld >= V, "greedy_next: bad sizes S=%lld V=%lld ld=%lld",
                (long long)S, (long long)V, (long long)ld);
  if (S == 0) return LSB_OK;
  LSB_CHECK_ARG(logits && tokens, "greedy_next: null pointer");
  LSB_CHECK_ARG(S <= 0x7fffffff && V <= 0x7fffffff, "greedy_next: shape too large");
  cudaStream_t st = (cudaStream_t)stream;
  return LSB_DISPATCH_DTYPE(dtype, T, [&] {
    LSB_CUDA_OK(lsb::launch_kernel(lsb::greedy_next_kernel<T>, dim3((unsigned)S), dim3(1024), 0, st,
                                   (const T*)logits, ld, (int)V, tokens, positions),
                "greedy_next");
    return LSB_OK;
  });
}
