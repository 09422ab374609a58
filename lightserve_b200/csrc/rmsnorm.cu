// Fused residual-add + RMSNorm (HBM-bound).
//
// Follows lightserve's _fused_add_rmsnorm_kernel
// (kernels/fused_rmsnorm_residual.py:31-70): h = x + residual is rounded to
// the input dtype and stored (:55-56); the mean of squares of float(h) is
// taken in fp32 (:64-65); out = float(h) * rrms * float(w) rounded to dtype
// (:68-70).
//
// B200 design: one CTA per row, the whole row held in registers as 16-byte
// vectors (128-bit LDG/STG, streaming loads since every byte is read once),
// so each row costs exactly 2 reads + 2 writes of M*N elements. The CTA width
// is chosen per N so that each thread owns VPT in {1,2,4,8} vectors. Rows that
// do not fit (N > 4096 vectors) or are not 16-byte aligned take a two-pass
// scalar kernel that re-reads h from the just-written h_out.
#include "common.cuh"

namespace lsb {

template <typename T, int VPT>
__global__ void __launch_bounds__(512)
rmsnorm_residual_vec_kernel(const T* __restrict__ x, const T* __restrict__ r,
                            const T* __restrict__ w, T* __restrict__ out,
                            T* __restrict__ h_out, int N, int64_t ld_x,
                            int64_t ld_r, int64_t ld_o, int64_t ld_h, float eps) {
  allow_dependents();
  wait_prerequisites();
  constexpr int VEC = Vec16<T>::N;
  const int row = blockIdx.x;
  const int nvec = N / VEC;
  const T* xr = x + row * ld_x;
  const T* rr = r + row * ld_r;

  Vec16<T> hv[VPT];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < nvec) {
      Vec16<T> a = ld_vec16_stream(xr + c * VEC);
      Vec16<T> b = ld_vec16_stream(rr + c * VEC);
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        T h = from_f<T>(to_f(a.v[j]) + to_f(b.v[j]));
        hv[i].v[j] = h;
        const float hf = to_f(h);
        ss = fmaf(hf, hf, ss);
      }
    }
  }

  __shared__ float red[16];
  ss = warp_sum(ss);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    float t = lane < nw ? red[lane] : 0.f;
    t = warp_sum(t);
    if (lane == 0) red[0] = t;
  }
  __syncthreads();
  const float rrms = 1.0f / sqrtf(red[0] / (float)N + eps);

  T* orow = out + row * ld_o;
  T* hrow = h_out + row * ld_h;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < nvec) {
      Vec16<T> wv = ld_vec16(w + c * VEC);
      Vec16<T> ov;
#pragma unroll
      for (int j = 0; j < VEC; ++j)
        ov.v[j] = from_f<T>(to_f(hv[i].v[j]) * rrms * to_f(wv.v[j]));
      __stcs(reinterpret_cast<uint4*>(hrow + c * VEC), *reinterpret_cast<uint4*>(&hv[i]));
      __stcs(reinterpret_cast<uint4*>(orow + c * VEC), *reinterpret_cast<uint4*>(&ov));
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256)
rmsnorm_residual_scalar_kernel(const T* __restrict__ x, const T* __restrict__ r,
                               const T* __restrict__ w, T* __restrict__ out,
                               T* __restrict__ h_out, int64_t N, int64_t ld_x,
                               int64_t ld_r, int64_t ld_o, int64_t ld_h, float eps) {
  const int64_t row = blockIdx.x;
  const T* xr = x + row * ld_x;
  const T* rr = r + row * ld_r;
  T* hrow = h_out + row * ld_h;
  float ss = 0.f;
  for (int64_t c = threadIdx.x; c < N; c += blockDim.x) {
    T h = from_f<T>(to_f(xr[c]) + to_f(rr[c]));
    hrow[c] = h;
    const float hf = to_f(h);
    ss = fmaf(hf, hf, ss);
  }
  __shared__ float red[8];
  ss = warp_sum(ss);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  if (warp == 0) {
    float t = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
    t = warp_sum(t);
    if (lane == 0) red[0] = t;
  }
  __syncthreads();
  const float rrms = 1.0f / sqrtf(red[0] / (float)N + eps);
  T* orow = out + row * ld_o;
  // Each thread re-reads only the h elements it wrote itself above.
  for (int64_t c = threadIdx.x; c < N; c += blockDim.x)
    orow[c] = from_f<T>(to_f(hrow[c]) * rrms * to_f(w[c]));
}

template <typename T>
static int launch_rmsnorm(const void* x, const void* r, const void* w, void* out,
                          void* h, int64_t M, int64_t N, int64_t ld_x, int64_t ld_r,
                          int64_t ld_o, int64_t ld_h, float eps, cudaStream_t st) {
  constexpr int VEC = Vec16<T>::N;
  const bool vec_ok = (N % VEC == 0) && aligned16(x) && aligned16(r) && aligned16(w) &&
                      aligned16(out) && aligned16(h) && (ld_x % VEC == 0) &&
                      (ld_r % VEC == 0) && (ld_o % VEC == 0) && (ld_h % VEC == 0) &&
                      (N / VEC) <= 512 * 8;
  if (M == 0 || N == 0) return LSB_OK;
  LSB_CHECK_ARG(M <= 0x7fffffff, "rmsnorm: M=%lld too large", (long long)M);
  if (vec_ok) {
    const int nvec = (int)(N / VEC);
    // Aim for ~4 vectors per thread, between 32 and 512 threads per row.
#ifndef LSB_RMS_VPT
#define LSB_RMS_VPT 2
#endif
    int threads = ((nvec + LSB_RMS_VPT - 1) / LSB_RMS_VPT + 31) / 32 * 32;
    threads = threads < 32 ? 32 : (threads > 512 ? 512 : threads);
    const int need = (nvec + threads - 1) / threads;
    const T* xp = (const T*)x; const T* rp = (const T*)r; const T* wp = (const T*)w;
    T* op = (T*)out; T* hp = (T*)h;
    dim3 grid((unsigned)M);
    if (need <= 1)
      LSB_CUDA_OK(launch_kernel(rmsnorm_residual_vec_kernel<T, 1>, grid, dim3(threads), 0, st, xp, rp, wp, op, hp, (int)N, ld_x, ld_r, ld_o, ld_h, eps), "rmsnorm_residual");
    else if (need <= 2)
      LSB_CUDA_OK(launch_kernel(rmsnorm_residual_vec_kernel<T, 2>, grid, dim3(threads), 0, st, xp, rp, wp, op, hp, (int)N, ld_x, ld_r, ld_o, ld_h, eps), "rmsnorm_residual");
    else if (need <= 4)
      LSB_CUDA_OK(launch_kernel(rmsnorm_residual_vec_kernel<T, 4>, grid, dim3(threads), 0, st, xp, rp, wp, op, hp, (int)N, ld_x, ld_r, ld_o, ld_h, eps), "rmsnorm_residual");
    else
      LSB_CUDA_OK(launch_kernel(rmsnorm_residual_vec_kernel<T, 8>, grid, dim3(threads), 0, st, xp, rp, wp, op, hp, (int)N, ld_x, ld_r, ld_o, ld_h, eps), "rmsnorm_residual");
  } else {
    rmsnorm_residual_scalar_kernel<T><<<(unsigned)M, 256, 0, st>>>(
        (const T*)x, (const T*)r, (const T*)w, (T*)out, (T*)h, N, ld_x, ld_r, ld_o, ld_h, eps);
  }
  LSB_CHECK_LAUNCH("rmsnorm_residual");
  return LSB_OK;
}

}  // namespace lsb

extern "C" int lsb_rmsnorm_residual(const void* x, const void* residual, const void* weight,
                                    void* out, void* h_out, int64_t M, int64_t N,
                                    int64_t ld_x, int64_t ld_r, int64_t ld_out, int64_t ld_h,
                                    float eps, int dtype, void* stream) {
  LSB_CHECK_ARG(M >= 0 && N >= 0, "rmsnorm: negative shape M=%lld N=%lld", (long long)M, (long long)N);
  LSB_CHECK_ARG((M == 0 || N == 0) || (x && residual && weight && out && h_out),
                "rmsnorm: null pointer");
  LSB_CHECK_ARG(ld_x >= N && ld_r >= N && ld_out >= N && ld_h >= N,
                "rmsnorm: row stride smaller than N");
  cudaStream_t st = (cudaStream_t)stream;
  return LSB_DISPATCH_DTYPE(dtype, T, [&] {
    return lsb::launch_rmsnorm<T>(x, residual, weight, out, h_out, M, N, ld_x, ld_r, ld_out,
                                  ld_h, eps, st);
  });
}
