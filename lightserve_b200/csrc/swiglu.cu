// Fused SwiGLU activation of the decode step's MLP (HBM/launch-bound).
//
// lightserve's Llama MLP computes F.silu(gate_proj(h)) * up_proj(h)
// (model/minimal_llama.py:231-233): silu runs in fp32 and rounds to the model
// dtype, then the product of the two dtype tensors is rounded again. This
// kernel does the same two roundings in one pass over the fused gate|up GEMM
// output gu = [S, 2I] (gate = gu[:, :I], up = gu[:, I:]) -> out = [S, I],
// replacing two elementwise launches and one intermediate tensor.
//
// One thread per 16-byte vector of out (8 bf16/fp16, 4 fp32); rows whose
// width or strides are not multiples of the vector take the scalar loop.
#include <algorithm>

#include "common.cuh"

namespace lsb {

template <typename T>
__device__ __forceinline__ T silu_mul(T g, T u) {
  const float x = to_f(g);
  const T s = from_f<T>(x / (1.0f + expf(-x)));  // F.silu in fp32, rounded to T
  return from_f<T>(to_f(s) * to_f(u));           // T * T, rounded to T
}

template <typename T>
__global__ void swiglu_vec_kernel(const T* __restrict__ gu, T* __restrict__ out, int64_t S,
                                  int64_t I, int64_t ld_gu, int64_t ld_out) {
  allow_dependents();
  wait_prerequisites();
  constexpr int VEC = Vec16<T>::N;
  const int64_t nv = I / VEC;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < S * nv;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = t / nv, c = (t - row * nv) * VEC;
    const Vec16<T> g = ld_vec16(gu + row * ld_gu + c);
    const Vec16<T> u = ld_vec16(gu + row * ld_gu + I + c);
    Vec16<T> o;
#pragma unroll
    for (int j = 0; j < VEC; ++j) o.v[j] = silu_mul(g.v[j], u.v[j]);
    st_vec16(out + row * ld_out + c, o);
  }
}

template <typename T>
__global__ void swiglu_scalar_kernel(const T* __restrict__ gu, T* __restrict__ out, int64_t S,
                                     int64_t I, int64_t ld_gu, int64_t ld_out) {
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < S * I;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = t / I, c = t - row * I;
    out[row * ld_out + c] = silu_mul(gu[row * ld_gu + c], gu[row * ld_gu + I + c]);
  }
}

template <typename T>
static int launch_swiglu(const void* gu, void* out, int64_t S, int64_t I, int64_t ld_gu,
                         int64_t ld_out, cudaStream_t st) {
  constexpr int VEC = Vec16<T>::N;
  const bool vec = I % VEC == 0 && ld_gu % VEC == 0 && ld_out % VEC == 0 && aligned16(gu) &&
                   aligned16(out);
  const int64_t work = vec ? S * (I / VEC) : S * I;
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((work + threads - 1) / threads, (int64_t)num_sms() * 8);
  if (vec)
    LSB_CUDA_OK(launch_kernel(swiglu_vec_kernel<T>, dim3((unsigned)blocks), dim3(threads), 0, st,
                              static_cast<const T*>(gu), static_cast<T*>(out), S, I, ld_gu, ld_out),
                "swiglu");
  else
    swiglu_scalar_kernel<T><<<(unsigned)blocks, threads, 0, st>>>(
        static_cast<const T*>(gu), static_cast<T*>(out), S, I, ld_gu, ld_out);
  LSB_CHECK_LAUNCH("swiglu");
  return LSB_OK;
}

}  // namespace lsb

extern "C" int lsb_swiglu(const void* gu, void* out, int64_t S, int64_t I, int64_t ld_gu,
                          int64_t ld_out, int dtype, void* stream) {
  LSB_CHECK_ARG(S >= 0 && I >= 0, "swiglu: negative shape S=%lld I=%lld", (long long)S, (long long)I);
  if (S == 0 || I == 0) return LSB_OK;
  LSB_CHECK_ARG(gu && out, "swiglu: null pointer");
  LSB_CHECK_ARG(ld_gu >= 2 * I && ld_out >= I, "swiglu: row stride too small");
  cudaStream_t st = (cudaStream_t)stream;
  return LSB_DISPATCH_DTYPE(dtype, T, [&] { return lsb::launch_swiglu<T>(gu, out, S, I, ld_gu, ld_out, st); });
}
