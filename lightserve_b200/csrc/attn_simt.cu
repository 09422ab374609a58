// CUDA-core (SIMT) FlashAttention forward and backward.
//
// This is the general-coverage path of the same extension: fp32 inputs (which
// lightserve's tests check at 1e-3 against an IEEE fp32 reference, so tensor
// cores with TF32 truncation are not allowed), any head dim up to 256, and
// arbitrary element strides. bf16/fp16 at head dims 64/128 with unit d-stride
// go to the tcgen05 kernel instead (attn_fwd_sm100.cu).
//
// Forward follows _flash_attn_fwd_kernel / _flash_attn_fwd_lse_kernel
// (kernels/flash_attention.py:84-179, kernels/flash_attention_backward.py:
// 88-169): scores s = (q.k) * scale, masked to -inf outside [0,N) and above
// the diagonal when causal, online softmax m/l/acc updates, P rounded to the
// input dtype before the PV product (kernels/flash_attention.py:168), output
// acc / l, and L = m + ln(l).
// Backward follows kernels/flash_attention_backward.py:202-330: Dsum =
// rowsum(dO*O) in fp32; per K/V tile a sweep over Q tiles recomputing
// P = exp(s - L); dV += P^T dO; dP = dO V^T; dS = P*(dP - Dsum) rounded to
// the input dtype; dK += dS^T Q * scale; dQ += dS K * scale accumulated in an
// fp32 buffer with atomics, then rounded to the input dtype.
#include "common.cuh"

namespace lsb {

struct Strides4 {
  int64_t b, h, n, d;
};

static inline Strides4 mk(const int64_t* s) { return Strides4{s[0], s[1], s[2], s[3]}; }

// ------------------------------------------------------------- forward ---

constexpr int FS_BM = 16;   // query rows per CTA
constexpr int FS_BN = 32;   // key rows per tile
constexpr int FS_THREADS = 128;

template <typename T>
__global__ void __launch_bounds__(FS_THREADS)
attn_fwd_simt_kernel(const T* __restrict__ q, const T* __restrict__ k,
                     const T* __restrict__ v, T* __restrict__ o, float* __restrict__ lse,
                     int H, int N, int D, int Dp, Strides4 sq, Strides4 sk, Strides4 sv,
                     Strides4 so, float scale, int causal) {
  extern __shared__ float smem[];
  float* Qs = smem;                   // [BM][Dp]
  float* Ks = Qs + FS_BM * Dp;        // [BN][Dp]
  float* Vs = Ks + FS_BN * Dp;        // [BN][Dp]
  float* Ps = Vs + FS_BN * Dp;        // [BM][BN]

  const int bh = blockIdx.y;
  const int b = bh / H, h = bh % H;
  const int m0 = blockIdx.x * FS_BM;
  const int tid = threadIdx.x;

  const T* qb = q + b * sq.b + h * sq.h;
  const T* kb = k + b * sk.b + h * sk.h;
  const T* vb = v + b * sv.b + h * sv.h;

  for (int i = tid; i < FS_BM * Dp; i += FS_THREADS) {
    const int r = i / Dp, d = i % Dp;
    const int m = m0 + r;
    Qs[i] = (m < N && d < D) ? to_f(qb[m * sq.n + d * sq.d]) : 0.f;
  }

  // Score mapping: row = tid / 8 (16 rows), 4 columns (tid % 8) * 4 + c.
  const int srow = tid >> 3;
  const int scol = (tid & 7) * 4;
  // Output mapping: the same row, d = (tid % 8) + 8 * j.
  const int dlane = tid & 7;
  float acc[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) acc[j] = 0.f;
  float m_i = -INFINITY, l_i = 0.f;

  const int hi = causal ? min(N, m0 + FS_BM) : N;
  for (int n0 = 0; n0 < hi; n0 += FS_BN) {
    __syncthreads();
    for (int i = tid; i < FS_BN * Dp; i += FS_THREADS) {
      const int r = i / Dp, d = i % Dp;
      const int n = n0 + r;
      const bool ok = n < N && d < D;
      Ks[i] = ok ? to_f(kb[n * sk.n + d * sk.d]) : 0.f;
      Vs[i] = ok ? to_f(vb[n * sv.n + d * sv.d]) : 0.f;
    }
    __syncthreads();

    float s[4];
    const int m = m0 + srow;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float* kr = Ks + (scol + c) * Dp;
      const float* qr = Qs + srow * Dp;
      float dot = 0.f;
      for (int d = 0; d < D; ++d) dot = fmaf(qr[d], kr[d], dot);
      const int n = n0 + scol + c;
      bool valid = (m < N) && (n < N);
      if (causal) valid = valid && (m >= n);
      s[c] = valid ? dot * scale : -INFINITY;
    }
    float mx = fmaxf(fmaxf(s[0], s[1]), fmaxf(s[2], s[3]));
#pragma unroll
    for (int off = 4; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    const float m_new = fmaxf(m_i, mx);
    // Rows with every score masked so far keep m = -inf; guard the exp.
    const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
    float p[4], psum = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      p[c] = expf(s[c] - m_use);
      psum += p[c];
    }
#pragma unroll
    for (int off = 4; off > 0; off >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
    const float alpha = expf(m_i - m_use);
    l_i = l_i * alpha + psum;
    m_i = m_new;
#pragma unroll
    for (int c = 0; c < 4; ++c)  // P is rounded to the input dtype before PV.
      Ps[srow * FS_BN + scol + c] = to_f(from_f<T>(p[c]));
    __syncwarp();
    __syncthreads();
    const float* pr = Ps + srow * FS_BN;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int d = dlane + 8 * j;
      if (d < Dp) {
        float a = acc[j] * alpha;
        for (int c = 0; c < FS_BN; ++c) a = fmaf(pr[c], Vs[c * Dp + d], a);
        acc[j] = a;
      }
    }
  }

  const int m = m0 + srow;
  if (m < N) {
    T* ob = o + b * so.b + h * so.h + m * so.n;
    const float inv = 1.0f / l_i;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int d = dlane + 8 * j;
      if (d < D) ob[d * so.d] = from_f<T>(acc[j] * inv);
    }
    if (lse != nullptr && dlane == 0) lse[((int64_t)b * H + h) * N + m] = m_i + logf(l_i);
  }
}

template <typename T>
static int launch_fwd_simt(const void* q, const void* k, const void* v, void* o, float* lse,
                           int64_t B, int64_t H, int64_t N, int64_t D, Strides4 sq,
                           Strides4 sk, Strides4 sv, Strides4 so, float scale, int causal,
                           cudaStream_t st) {
  const int Dp = (int)((D + 7) / 8 * 8);
  const size_t smem = sizeof(float) * (size_t)(FS_BM * Dp + 2 * FS_BN * Dp + FS_BM * FS_BN);
  static SmemLimit smem_limit;
  if (int rc_ = smem_limit.ensure(attn_fwd_simt_kernel<T>, smem, "attn_fwd_simt smem attribute")) return rc_;
  dim3 grid((unsigned)((N + FS_BM - 1) / FS_BM), (unsigned)(B * H));
  attn_fwd_simt_kernel<T><<<grid, FS_THREADS, smem, st>>>(
      (const T*)q, (const T*)k, (const T*)v, (T*)o, lse, (int)H, (int)N, (int)D, Dp, sq, sk, sv,
      so, scale, causal);
  LSB_CHECK_LAUNCH("attn_fwd_simt");
  return LSB_OK;
}

// ------------------------------------------------------------ backward ---

constexpr int BS_BN = 16;  // key rows per CTA
constexpr int BS_BM = 32;  // query rows per inner step
constexpr int BS_THREADS = 128;

template <typename T>
__global__ void __launch_bounds__(BS_THREADS)
attn_bwd_simt_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                     const T* __restrict__ dout, const float* __restrict__ lse,
                     const float* __restrict__ dsum, float* __restrict__ dq_acc,
                     T* __restrict__ dk, T* __restrict__ dv, int H, int N, int D, int Dp,
                     Strides4 sq, Strides4 sk, Strides4 sv, Strides4 sdo, Strides4 sdk,
                     Strides4 sdv, float scale, int causal) {
  extern __shared__ float smem[];
  float* Ks = smem;                 // [BN][Dp]
  float* Vs = Ks + BS_BN * Dp;      // [BN][Dp]
  float* Qs = Vs + BS_BN * Dp;      // [BM][Dp]
  float* dOs = Qs + BS_BM * Dp;     // [BM][Dp]
  float* Ps = dOs + BS_BM * Dp;     // [BM][BN]
  float* dSs = Ps + BS_BM * BS_BN;  // [BM][BN]
  float* Ls = dSs + BS_BM * BS_BN;  // [BM]
  float* Ds = Ls + BS_BM;           // [BM]

  const int bh = blockIdx.y;
  const int b = bh / H, h = bh % H;
  const int n0 = blockIdx.x * BS_BN;
  const int tid = threadIdx.x;

  const T* qb = q + b * sq.b + h * sq.h;
  const T* kb = k + b * sk.b + h * sk.h;
  const T* vb = v + b * sv.b + h * sv.h;
  const T* dob = dout + b * sdo.b + h * sdo.h;
  const float* lb = lse + (int64_t)bh * N;
  const float* db = dsum + (int64_t)bh * N;
  float* dqb = dq_acc + (int64_t)bh * N * D;

  for (int i = tid; i < BS_BN * Dp; i += BS_THREADS) {
    const int r = i / Dp, d = i % Dp;
    const int n = n0 + r;
    const bool ok = n < N && d < D;
    Ks[i] = ok ? to_f(kb[n * sk.n + d * sk.d]) : 0.f;
    Vs[i] = ok ? to_f(vb[n * sv.n + d * sv.d]) : 0.f;
  }

  // dK/dV mapping: key row tid / 8, d = (tid % 8) + 8 j.
  const int krow = tid >> 3, dl8 = tid & 7;
  float dk_acc[32], dv_acc[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) { dk_acc[j] = 0.f; dv_acc[j] = 0.f; }

  // Score mapping: query row tid / 4, key columns (tid % 4) * 4 + c.
  const int srow = tid >> 2, scol = (tid & 3) * 4;

  // Causal: query tiles entirely above this key tile's diagonal contribute 0.
  const int lo = causal ? (n0 / BS_BM) * BS_BM : 0;
  for (int m0 = lo; m0 < N; m0 += BS_BM) {
    __syncthreads();
    for (int i = tid; i < BS_BM * Dp; i += BS_THREADS) {
      const int r = i / Dp, d = i % Dp;
      const int m = m0 + r;
      const bool ok = m < N && d < D;
      Qs[i] = ok ? to_f(qb[m * sq.n + d * sq.d]) : 0.f;
      dOs[i] = ok ? to_f(dob[m * sdo.n + d * sdo.d]) : 0.f;
    }
    if (tid < BS_BM) {
      const int m = m0 + tid;
      Ls[tid] = m < N ? lb[m] : 0.f;
      Ds[tid] = m < N ? db[m] : 0.f;
    }
    __syncthreads();

    const int m = m0 + srow;
    const float* qr = Qs + srow * Dp;
    const float* dor = dOs + srow * Dp;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int kc = scol + c;
      const int n = n0 + kc;
      const float* kr = Ks + kc * Dp;
      const float* vr = Vs + kc * Dp;
      float s = 0.f, dp = 0.f;
      for (int d = 0; d < D; ++d) {
        s = fmaf(qr[d], kr[d], s);
        dp = fmaf(dor[d], vr[d], dp);
      }
      bool valid = (m < N) && (n < N);
      if (causal) valid = valid && (m >= n);
      const float p = valid ? expf(s * scale - Ls[srow]) : 0.f;
      const float ds = p * (dp - Ds[srow]);
      Ps[srow * BS_BN + kc] = to_f(from_f<T>(p));   // P cast to the dO dtype for dV
      dSs[srow * BS_BN + kc] = to_f(from_f<T>(ds)); // dS cast to the q dtype
    }
    __syncthreads();

    // dV[krow][d] += sum_m P[m][krow] dO[m][d];  dK[krow][d] += sum_m dS[m][krow] Q[m][d]
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int d = dl8 + 8 * j;
      if (d < Dp) {
        float av = dv_acc[j], ak = dk_acc[j];
        for (int mm = 0; mm < BS_BM; ++mm) {
          av = fmaf(Ps[mm * BS_BN + krow], dOs[mm * Dp + d], av);
          ak = fmaf(dSs[mm * BS_BN + krow], Qs[mm * Dp + d], ak);
        }
        dv_acc[j] = av;
        dk_acc[j] = ak;
      }
    }

    // dQ[m][d] += scale * sum_k dS[m][k] K[k][d]   (fp32 atomics)
    if (m < N) {
      const float* dsr = dSs + srow * BS_BN;
      for (int d = (tid & 3); d < D; d += 4) {
        float a = 0.f;
#pragma unroll
        for (int kc = 0; kc < BS_BN; ++kc) a = fmaf(dsr[kc], Ks[kc * Dp + d], a);
        atomicAdd(dqb + (int64_t)m * D + d, a * scale);
      }
    }
  }

  const int n = n0 + krow;
  if (n < N) {
    T* dkr = dk + b * sdk.b + h * sdk.h + n * sdk.n;
    T* dvr = dv + b * sdv.b + h * sdv.h + n * sdv.n;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int d = dl8 + 8 * j;
      if (d < D) {
        dkr[d * sdk.d] = from_f<T>(dk_acc[j] * scale);
        dvr[d * sdv.d] = from_f<T>(dv_acc[j]);
      }
    }
  }
}

// dq = dq_acc (fp32, [B,H,N,D] contiguous) rounded to the input dtype.
template <typename T>
__global__ void attn_dq_cast_kernel(const float* __restrict__ dq_acc, T* __restrict__ dq, int H,
                                    int N, int D, Strides4 sdq, int64_t total) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int d = (int)(i % D);
    const int64_t r = i / D;
    const int m = (int)(r % N);
    const int bh = (int)(r / N);
    const int b = bh / H, h = bh % H;
    dq[b * sdq.b + h * sdq.h + m * sdq.n + d * sdq.d] = from_f<T>(dq_acc[i]);
  }
}

// Dsum[b,h,m] = sum_d float(dO) * float(O)   (kernels/flash_attention_backward.py:202-229)
template <typename T>
__global__ void attn_dsum_rows_kernel(const T* __restrict__ o, const T* __restrict__ dout,
                                      float* __restrict__ dsum, int H, int N, int D,
                                      Strides4 so, Strides4 sdo, int64_t rows) {
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const int bh = (int)(warp / N), m = (int)(warp % N);
  const int b = bh / H, h = bh % H;
  const T* orow = o + b * so.b + h * so.h + m * so.n;
  const T* drow = dout + b * sdo.b + h * sdo.h + m * sdo.n;
  float acc = 0.f;
  for (int d = lane; d < D; d += 32) acc = fmaf(to_f(orow[d * so.d]), to_f(drow[d * sdo.d]), acc);
  acc = warp_sum(acc);
  if (lane == 0) dsum[warp] = acc;
}

// Vectorised Dsum for unit d-stride, 16-byte aligned rows: LPR lanes read one
// row with 16-byte loads; 32 / LPR rows per warp.
template <typename T, int LPR>
__global__ void __launch_bounds__(256)
attn_dsum_vec_kernel(const T* __restrict__ o, const T* __restrict__ dout, float* __restrict__ dsum,
                     int H, int N, Strides4 so, Strides4 sdo, int64_t rows,
                     float* __restrict__ zero_rows, int* __restrict__ zero_counter) {
  constexpr int VEC = 16 / sizeof(T);
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / LPR;
  const int sub = threadIdx.x % LPR;
  const bool ok = row < rows;
  float acc = 0.f;
  if (ok) {
    const int bh = (int)(row / N), m = (int)(row % N);
    const int b = bh / H, h = bh % H;
    Vec16<T> a = ld_vec16_stream(o + b * so.b + h * so.h + m * so.n + sub * VEC);
    Vec16<T> c = ld_vec16_stream(dout + b * sdo.b + h * sdo.h + m * sdo.n + sub * VEC);
#pragma unroll
    for (int j = 0; j < VEC; ++j) acc = fmaf(to_f(a.v[j]), to_f(c.v[j]), acc);
    if (zero_rows != nullptr) {
      // The same row of the dense fp32 dQ accumulator ([rows][LPR * VEC]).
      float4* z = reinterpret_cast<float4*>(zero_rows + row * (LPR * VEC)) + sub * (VEC / 4);
#pragma unroll
      for (int j = 0; j < VEC / 4; ++j) z[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  if (zero_counter != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *zero_counter = 0;
#pragma unroll
  for (int off = LPR / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (ok && sub == 0) dsum[row] = acc;
}

// Vectorised dQ cast for a dense [B,H,N,D] output: 8 fp32 -> 8 x 16-bit per thread.
template <typename T>
__global__ void attn_dq_cast_vec_kernel(const float4* __restrict__ src, uint4* __restrict__ dst,
                                        int64_t n8) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float4 a = __ldcs(src + 2 * i), b = __ldcs(src + 2 * i + 1);
    Vec16<T> v;
    v.v[0] = from_f<T>(a.x); v.v[1] = from_f<T>(a.y); v.v[2] = from_f<T>(a.z); v.v[3] = from_f<T>(a.w);
    v.v[4] = from_f<T>(b.x); v.v[5] = from_f<T>(b.y); v.v[6] = from_f<T>(b.z); v.v[7] = from_f<T>(b.w);
    __stcs(dst + i, *reinterpret_cast<uint4*>(&v));
  }
}

// Dsum pass. When zero_rows is given (the dense fp32 dQ accumulator) and
// the vectorised kernel applies, the same launch zeroes it and *zero_counter
// (the backward kernel's work counter) and sets *zeroed; the caller zeroes
// them itself otherwise.
template <typename T>
int launch_dsum(const void* o, const void* dout, float* dsum, int64_t B, int64_t H, int64_t N,
                int64_t D, Strides4 so, Strides4 sdo, cudaStream_t st, float* zero_rows,
                int* zero_counter, bool* zeroed) {
  const int64_t rows = B * H * N;
  const int threads = 256;
  constexpr int VEC = 16 / sizeof(T);
  if (zeroed) *zeroed = false;
  const bool vec = so.d == 1 && sdo.d == 1 && aligned16(o) && aligned16(dout) &&
                   (so.n * sizeof(T)) % 16 == 0 && (so.h * sizeof(T)) % 16 == 0 &&
                   (so.b * sizeof(T)) % 16 == 0 && (sdo.n * sizeof(T)) % 16 == 0 &&
                   (sdo.h * sizeof(T)) % 16 == 0 && (sdo.b * sizeof(T)) % 16 == 0;
  if (vec && (D == 16 * VEC || D == 8 * VEC)) {
    const int lpr = (int)(D / VEC);
    const int64_t blocks = (rows * lpr + threads - 1) / threads;
    float* z = (zero_rows != nullptr && aligned16(zero_rows)) ? zero_rows : nullptr;
    int* zc = z != nullptr ? zero_counter : nullptr;
    if (lpr == 16)
      attn_dsum_vec_kernel<T, 16><<<(unsigned)blocks, threads, 0, st>>>(
          (const T*)o, (const T*)dout, dsum, (int)H, (int)N, so, sdo, rows, z, zc);
    else
      attn_dsum_vec_kernel<T, 8><<<(unsigned)blocks, threads, 0, st>>>(
          (const T*)o, (const T*)dout, dsum, (int)H, (int)N, so, sdo, rows, z, zc);
    LSB_CHECK_LAUNCH("attn_bwd_dsum");
    if (zeroed) *zeroed = z != nullptr;
    return LSB_OK;
  }
  const int64_t blocks = (rows * 32 + threads - 1) / threads;
  attn_dsum_rows_kernel<T><<<(unsigned)blocks, threads, 0, st>>>(
      (const T*)o, (const T*)dout, dsum, (int)H, (int)N, (int)D, so, sdo, rows);
  LSB_CHECK_LAUNCH("attn_bwd_dsum");
  return LSB_OK;
}

template <typename T>
int launch_dq_cast(const float* dq_acc, void* dq, int64_t B, int64_t H, int64_t N, int64_t D,
                   Strides4 sdq, cudaStream_t st) {
  const int64_t total = B * H * N * D;
  const bool dense = sdq.d == 1 && sdq.n == D && sdq.h == N * D && sdq.b == H * N * D;
  if (sizeof(T) == 2 && dense && total % 8 == 0 && aligned16(dq) && aligned16(dq_acc)) {
    const int64_t n8 = total / 8;
    int64_t blocks = (n8 + 255) / 256;
    const int64_t cap = (int64_t)num_sms() * 16;
    if (blocks > cap) blocks = cap;
    attn_dq_cast_vec_kernel<T><<<(unsigned)blocks, 256, 0, st>>>(
        reinterpret_cast<const float4*>(dq_acc), reinterpret_cast<uint4*>(dq), n8);
    LSB_CHECK_LAUNCH("attn_dq_cast");
    return LSB_OK;
  }
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  attn_dq_cast_kernel<T><<<(unsigned)blocks, 256, 0, st>>>(dq_acc, (T*)dq, (int)H, (int)N,
                                                           (int)D, sdq, total);
  LSB_CHECK_LAUNCH("attn_dq_cast");
  return LSB_OK;
}

template <typename T>
static int launch_bwd_simt(const void* q, const void* k, const void* v, const void* o,
                           const void* dout, const float* lse, void* dq, void* dk, void* dv,
                           int64_t B, int64_t H, int64_t N, int64_t D, Strides4 sq, Strides4 sk,
                           Strides4 sv, Strides4 so, Strides4 sdo, Strides4 sdq, Strides4 sdk,
                           Strides4 sdv, float scale, int causal, float* dsum, float* dq_acc,
                           cudaStream_t st) {
  bool zeroed = false;
  int rc = launch_dsum<T>(o, dout, dsum, B, H, N, D, so, sdo, st, dq_acc, nullptr, &zeroed);
  if (rc) return rc;
  if (!zeroed)
    LSB_CUDA_OK(cudaMemsetAsync(dq_acc, 0, sizeof(float) * (size_t)(B * H * N * D), st),
                "attn_bwd dQ accumulator memset");
  const int Dp = (int)((D + 7) / 8 * 8);
  const size_t smem =
      sizeof(float) * (size_t)(2 * BS_BN * Dp + 2 * BS_BM * Dp + 2 * BS_BM * BS_BN + 2 * BS_BM);
  static SmemLimit smem_limit;
  if (int rc_ = smem_limit.ensure(attn_bwd_simt_kernel<T>, smem, "attn_bwd_simt smem attribute")) return rc_;
  dim3 grid((unsigned)((N + BS_BN - 1) / BS_BN), (unsigned)(B * H));
  attn_bwd_simt_kernel<T><<<grid, BS_THREADS, smem, st>>>(
      (const T*)q, (const T*)k, (const T*)v, (const T*)dout, lse, dsum, dq_acc, (T*)dk, (T*)dv,
      (int)H, (int)N, (int)D, Dp, sq, sk, sv, sdo, sdk, sdv, scale, causal);
  LSB_CHECK_LAUNCH("attn_bwd_simt");
  return launch_dq_cast<T>(dq_acc, dq, B, H, N, D, sdq, st);
}

// Explicit instantiations used by the tcgen05 backward path (attn_bwd_sm100.cu).
template int launch_dsum<__nv_bfloat16>(const void*, const void*, float*, int64_t, int64_t,
                                        int64_t, int64_t, Strides4, Strides4, cudaStream_t,
                                        float*, int*, bool*);
template int launch_dsum<__half>(const void*, const void*, float*, int64_t, int64_t, int64_t,
                                 int64_t, Strides4, Strides4, cudaStream_t, float*, int*, bool*);
template int launch_dq_cast<__nv_bfloat16>(const float*, void*, int64_t, int64_t, int64_t,
                                           int64_t, Strides4, cudaStream_t);
template int launch_dq_cast<__half>(const float*, void*, int64_t, int64_t, int64_t, int64_t,
                                    Strides4, cudaStream_t);

int attn_fwd_simt(const void* q, const void* k, const void* v, void* o, float* lse, int64_t B,
                  int64_t H, int64_t N, int64_t D, const int64_t* sq, const int64_t* sk,
                  const int64_t* sv, const int64_t* so, float scale, int causal, int dtype,
                  cudaStream_t st) {
  LSB_CHECK_ARG(D <= 256, "attn_fwd (SIMT): head dim %lld > 256 unsupported", (long long)D);
  return LSB_DISPATCH_DTYPE(dtype, T, [&] {
    return launch_fwd_simt<T>(q, k, v, o, lse, B, H, N, D, mk(sq), mk(sk), mk(sv), mk(so), scale,
                              causal, st);
  });
}

int attn_bwd_simt(const void* q, const void* k, const void* v, const void* o, const void* dout,
                  const float* lse, void* dq, void* dk, void* dv, int64_t B, int64_t H, int64_t N,
                  int64_t D, const int64_t* sq, const int64_t* sk, const int64_t* sv,
                  const int64_t* so, const int64_t* sdo, const int64_t* sdq, const int64_t* sdk,
                  const int64_t* sdv, float scale, int causal, int dtype, float* dsum,
                  float* dq_acc, cudaStream_t st) {
  LSB_CHECK_ARG(D <= 256, "attn_bwd (SIMT): head dim %lld > 256 unsupported", (long long)D);
  return LSB_DISPATCH_DTYPE(dtype, T, [&] {
    return launch_bwd_simt<T>(q, k, v, o, dout, lse, dq, dk, dv, B, H, N, D, mk(sq), mk(sk),
                              mk(sv), mk(so), mk(sdo), mk(sdq), mk(sdk), mk(sdv), scale, causal,
                              dsum, dq_acc, st);
  });
}

}  // namespace lsb
