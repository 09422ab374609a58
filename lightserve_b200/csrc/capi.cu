// C ABI entry points that dispatch between kernels, plus error reporting.
#include "common.cuh"

#include <string.h>

namespace lsb {

static thread_local char g_err[512] = {0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

// attn_simt.cu
int attn_fwd_simt(const void* q, const void* k, const void* v, void* o, float* lse, int64_t B,
                  int64_t H, int64_t N, int64_t D, const int64_t* sq, const int64_t* sk,
                  const int64_t* sv, const int64_t* so, float scale, int causal, int dtype,
                  cudaStream_t st);
int attn_bwd_simt(const void* q, const void* k, const void* v, const void* o, const void* dout,
                  const float* lse, void* dq, void* dk, void* dv, int64_t B, int64_t H, int64_t N,
                  int64_t D, const int64_t* sq, const int64_t* sk, const int64_t* sv,
                  const int64_t* so, const int64_t* sdo, const int64_t* sdq, const int64_t* sdk,
                  const int64_t* sdv, float scale, int causal, int dtype, float* dsum,
                  float* dq_acc, cudaStream_t st);
// attn_fwd_sm100.cu
bool attn_fwd_tc_eligible(const void* q, const void* k, const void* v, const void* o, int64_t B,
                          int64_t H, int64_t N, int64_t D, const int64_t* sq, const int64_t* sk,
                          const int64_t* sv, const int64_t* so, int dtype);
int attn_fwd_tc(const void* q, const void* k, const void* v, void* o, float* lse, int64_t B,
                int64_t H, int64_t N, int64_t D, const int64_t* sq, const int64_t* sk,
                const int64_t* sv, const int64_t* so, float scale, int causal, int dtype,
                cudaStream_t st);
int attn_fwd_varlen_tc(const void* q, const void* k, const void* v, void* o, float* lse,
                       const int* cu_seqlens, int64_t n_seqs, int64_t max_seqlen, int64_t T,
                       int64_t H, int64_t D, const int64_t* sq, const int64_t* sk,
                       const int64_t* sv, const int64_t* so, float scale, int causal, int dtype,
                       cudaStream_t st);
// attn_bwd_sm100.cu
bool attn_bwd_tc_eligible(const void* q, const void* k, const void* v, const void* o,
                          const void* dout, const void* dq, const void* dk, const void* dv,
                          int64_t B, int64_t H, int64_t N, int64_t D, const int64_t* sq,
                          const int64_t* sk, const int64_t* sv, const int64_t* so,
                          const int64_t* sdo, const int64_t* sdq, const int64_t* sdk,
                          const int64_t* sdv, int dtype);
int attn_bwd_tc(const void* q, const void* k, const void* v, const void* o, const void* dout,
                const float* lse, void* dq, void* dk, void* dv, int64_t B, int64_t H, int64_t N,
                int64_t D, const int64_t* sq, const int64_t* sk, const int64_t* sv,
                const int64_t* so, const int64_t* sdo, const int64_t* sdq, const int64_t* sdk,
                const int64_t* sdv, float scale, int causal, int dtype, float* dsum,
                float* dq_acc, cudaStream_t st);

int attn_fwd_tc_device_error(bool reset);
int attn_bwd_tc_device_error(bool reset);
int paged_decode_device_error(bool reset);
int selftest_device_error(bool reset);
int linear_device_error(bool reset);


}  // namespace lsb

extern "C" const char* lsb_last_error(void) { return lsb::g_err; }

namespace lsb {
static std::atomic<int> g_programmatic_launch{1};
bool programmatic_launch() { return g_programmatic_launch.load(std::memory_order_relaxed) != 0; }
}  // namespace lsb

extern "C" int lsb_set_programmatic_launch(int enable) {
  return lsb::g_programmatic_launch.exchange(enable ? 1 : 0);
}

static int device_error_all(bool reset) {
  int e = 0;
  for (int v : {lsb::attn_fwd_tc_device_error(reset), lsb::attn_bwd_tc_device_error(reset),
                lsb::paged_decode_device_error(reset), lsb::selftest_device_error(reset),
                lsb::linear_device_error(reset)})
    if (!e) e = v;
  if (e == LSB_DEVICE_ERR_QUERY)
    lsb::set_error("device error words unreadable: %s", cudaGetErrorString(cudaGetLastError()));
  return e;
}

extern "C" int lsb_device_error(void) { return device_error_all(false); }

extern "C" int lsb_device_error_reset(void) { return device_error_all(true); }

extern "C" const char* lsb_version(void) { return "lightserve_b200 0.1 (sm_100a)"; }

static int check_attn_common(const char* who, int64_t B, int64_t H, int64_t N, int64_t D,
                             int dtype) {
  LSB_CHECK_ARG(B >= 0 && H >= 0 && N >= 0 && D > 0, "%s: bad shape B=%lld H=%lld N=%lld D=%lld",
                who, (long long)B, (long long)H, (long long)N, (long long)D);
  LSB_CHECK_ARG(lsb::dtype_size(dtype) > 0, "%s: unsupported dtype %d", who, dtype);
  LSB_CHECK_ARG(B * H <= 0x7fffffffLL && N <= 0x7fffffffLL, "%s: shape too large", who);
  return LSB_OK;
}

extern "C" int lsb_attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
                            int64_t B, int64_t H, int64_t N, int64_t D, const int64_t* sq,
                            const int64_t* sk, const int64_t* sv, const int64_t* so, float scale,
                            int causal, int dtype, int impl, void* stream) {
  int rc = check_attn_common("attn_fwd", B, H, N, D, dtype);
  if (rc) return rc;
  if (B == 0 || H == 0 || N == 0) return LSB_OK;
  LSB_CHECK_ARG(q && k && v && o && sq && sk && sv && so, "attn_fwd: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const bool tc_ok = lsb::attn_fwd_tc_eligible(q, k, v, o, B, H, N, D, sq, sk, sv, so, dtype);
  if (impl == LSB_IMPL_TCGEN05 || (impl == LSB_IMPL_AUTO && tc_ok)) {
    LSB_CHECK_ARG(tc_ok,
                  "attn_fwd: tcgen05 kernel needs bf16/fp16, D in {64,128}, unit d-stride and "
                  "16-byte aligned strides");
    return lsb::attn_fwd_tc(q, k, v, o, lse, B, H, N, D, sq, sk, sv, so, scale, causal, dtype, st);
  }
  LSB_CHECK_ARG(impl == LSB_IMPL_AUTO || impl == LSB_IMPL_SIMT, "attn_fwd: bad impl %d", impl);
  return lsb::attn_fwd_simt(q, k, v, o, lse, B, H, N, D, sq, sk, sv, so, scale, causal, dtype, st);
}

extern "C" int lsb_attn_fwd_varlen(const void* q, const void* k, const void* v, void* o,
                                   float* lse, const int32_t* cu_seqlens, int64_t num_seqs,
                                   int64_t max_seqlen, int64_t total_tokens, int64_t H, int64_t D,
                                   const int64_t* sq, const int64_t* sk, const int64_t* sv,
                                   const int64_t* so, float scale, int causal, int dtype,
                                   void* stream) {
  int rc = check_attn_common("attn_fwd_varlen", num_seqs, H, total_tokens, D, dtype);
  if (rc) return rc;
  LSB_CHECK_ARG(max_seqlen >= 0 && max_seqlen <= total_tokens,
                "attn_fwd_varlen: max_seqlen %lld outside [0, total_tokens=%lld]",
                (long long)max_seqlen, (long long)total_tokens);
  if (num_seqs == 0 || H == 0 || total_tokens == 0 || max_seqlen == 0) return LSB_OK;
  LSB_CHECK_ARG(q && k && v && o && cu_seqlens && sq && sk && sv && so,
                "attn_fwd_varlen: null pointer");
  // The packed [T, H, D] tensors are checked as [1, H, T, D] with strides
  // {0, head, token, 1}.
  const int64_t q4[4] = {0, sq[1], sq[0], 1}, k4[4] = {0, sk[1], sk[0], 1};
  const int64_t v4[4] = {0, sv[1], sv[0], 1}, o4[4] = {0, so[1], so[0], 1};
  LSB_CHECK_ARG(sq[2] == 1 && sk[2] == 1 && sv[2] == 1 && so[2] == 1 &&
                    lsb::attn_fwd_tc_eligible(q, k, v, o, 1, H, total_tokens, D, q4, k4, v4, o4,
                                              dtype),
                "attn_fwd_varlen: needs bf16/fp16, D in {64,128}, unit d-stride and 16-byte "
                "aligned token / head strides");
  return lsb::attn_fwd_varlen_tc(q, k, v, o, lse, cu_seqlens, num_seqs, max_seqlen, total_tokens,
                                 H, D, sq, sk, sv, so, scale, causal, dtype,
                                 (cudaStream_t)stream);
}

extern "C" int64_t lsb_attn_bwd_workspace_size(int64_t B, int64_t H, int64_t N, int64_t D) {
  if (B <= 0 || H <= 0 || N <= 0 || D <= 0) return 0;
  // Dsum, dQ accumulator, and the tcgen05 kernel's work-item counter.
  return lsb::align256(4 * B * H * N) + lsb::align256(4 * B * H * N * D) + 256;
}

extern "C" int lsb_attn_bwd(const void* q, const void* k, const void* v, const void* o,
                            const void* dout, const float* lse, void* dq, void* dk, void* dv,
                            int64_t B, int64_t H, int64_t N, int64_t D, const int64_t* sq,
                            const int64_t* sk, const int64_t* sv, const int64_t* so,
                            const int64_t* sdo, const int64_t* sdq, const int64_t* sdk,
                            const int64_t* sdv, float scale, int causal, int dtype, int impl,
                            void* workspace, int64_t workspace_bytes, void* stream) {
  int rc = check_attn_common("attn_bwd", B, H, N, D, dtype);
  if (rc) return rc;
  if (B == 0 || H == 0 || N == 0) return LSB_OK;
  LSB_CHECK_ARG(q && k && v && o && dout && lse && dq && dk && dv, "attn_bwd: null pointer");
  const int64_t need = lsb_attn_bwd_workspace_size(B, H, N, D);
  LSB_CHECK_ARG(workspace && workspace_bytes >= need && (((uintptr_t)workspace) & 255) == 0,
                "attn_bwd: workspace of %lld bytes (256-byte aligned) required, got %lld",
                (long long)need, (long long)workspace_bytes);
  float* dsum = (float*)workspace;
  float* dq_acc = (float*)((char*)workspace + lsb::align256(4 * B * H * N));
  cudaStream_t st = (cudaStream_t)stream;
  const bool tc_ok = lsb::attn_bwd_tc_eligible(q, k, v, o, dout, dq, dk, dv, B, H, N, D, sq, sk,
                                               sv, so, sdo, sdq, sdk, sdv, dtype);
  if (impl == LSB_IMPL_TCGEN05 || (impl == LSB_IMPL_AUTO && tc_ok)) {
    LSB_CHECK_ARG(tc_ok, "attn_bwd: tcgen05 kernel not eligible for these inputs");
    return lsb::attn_bwd_tc(q, k, v, o, dout, lse, dq, dk, dv, B, H, N, D, sq, sk, sv, so, sdo,
                            sdq, sdk, sdv, scale, causal, dtype, dsum, dq_acc, st);
  }
  LSB_CHECK_ARG(impl == LSB_IMPL_AUTO || impl == LSB_IMPL_SIMT, "attn_bwd: bad impl %d", impl);
  return lsb::attn_bwd_simt(q, k, v, o, dout, lse, dq, dk, dv, B, H, N, D, sq, sk, sv, so, sdo,
                            sdq, sdk, sdv, scale, causal, dtype, dsum, dq_acc, st);
}
