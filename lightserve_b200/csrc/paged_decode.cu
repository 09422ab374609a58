// Paged-KV decode attention and the KV-cache write (HBM-bound).
//
// lightserve has no decode-shaped attention kernel (engine/README.md:142-147);
// its decode re-runs the full causal forward every step
// (model/cuda_graph_decode.py:108-149). These kernels compute the same
// attention row -- the newest position attending to every cached position
// 0..L-1 of its own sequence, which is the last row of the causal mask -- from
// a paged cache addressed through engine/block_manager.py's block tables
// (block i of a request holds tokens [i*block_size, (i+1)*block_size),
// engine/block_manager.py:58-61).
//
// Cache layout: [num_blocks, H, block_size, D] per layer, so one (block, head)
// is a contiguous block_size*D run (4 KiB for bf16, 16 x 128): each half-warp
// reads a whole 256-byte token row with 16-byte loads.
//
// Decode kernel (flash-decoding): grid (partition, head, sequence). Each CTA
// covers PART_TOKENS cached tokens of one (sequence, head); its 4 warps take
// interleaved rounds of 16 tokens, issue all K and V loads of a round before
// any math (16 x 16 B in flight per lane), and keep an online softmax in fp32
// with exp2 on log2(e)-prescaled scores. Sequences with one partition write
// the output directly; longer ones write (m, l, acc) partials to the
// caller-provided workspace and a combine kernel merges them.
#include "common.cuh"
#include "sm100.cuh"

#include <mutex>
#include <type_traits>

namespace lsb {

constexpr int PD_PART_TOKENS = 512;
constexpr int PD_WARPS = 4;
constexpr float PD_LOG2E = 1.4426950408889634f;

static inline int64_t pd_max_parts(int64_t max_blocks, int64_t bs) {
  const int64_t max_tokens = max_blocks * bs;
  return (max_tokens + PD_PART_TOKENS - 1) / PD_PART_TOKENS;
}

// Workspace: part_m [S*H*P], part_l [S*H*P], part_acc [S*H*P*D] (fp32).
template <typename T, int D>
__global__ void __launch_bounds__(PD_WARPS * 32)
paged_decode_kernel(const T* __restrict__ q, const T* __restrict__ k_cache,
                    const T* __restrict__ v_cache, const int32_t* __restrict__ block_tables,
                    const int32_t* __restrict__ context_lens, T* __restrict__ o, int H,
                    int max_blocks, int num_blocks, int bs_log2, int64_t sq_s, int64_t sq_h, int64_t so_s,
                    int64_t so_h, float scale_log2, int max_parts, float* __restrict__ part_m,
                    float* __restrict__ part_l, float* __restrict__ part_acc) {
  constexpr int VEC = 16 / sizeof(T);
  constexpr int LPT = D / VEC;         // lanes per token row
  constexpr int TPW = 32 / LPT;        // token rows per warp-wide load
  constexpr int U = (16 / TPW) > 0 ? (16 / TPW) : 1;  // loads per lane per round
  constexpr int ROUND = TPW * U;       // tokens per warp round
  static_assert(LPT >= 1 && LPT <= 32 && (32 % LPT) == 0, "unsupported head dim");

  const int part = blockIdx.x, h = blockIdx.y, s = blockIdx.z;
  // Positions past the block table's capacity are never read.
  const int ctx = max(0, min(context_lens[s], max_blocks << bs_log2));
  const int t_begin = part * PD_PART_TOKENS;
  if (t_begin >= ctx && !(ctx == 0 && part == 0)) return;
  const int t_end = min(ctx, t_begin + PD_PART_TOKENS);
  const int nparts = (ctx + PD_PART_TOKENS - 1) / PD_PART_TOKENS;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = lane / LPT;          // which token row of a load this lane reads
  const int dofs = (lane % LPT) * VEC; // which 16-byte chunk of that row

  float qf[VEC];
  {
    Vec16<T> qv = ld_vec16(q + s * sq_s + h * sq_h + dofs);
#pragma unroll
    for (int j = 0; j < VEC; ++j) qf[j] = to_f(qv.v[j]) * scale_log2;
  }

  const int32_t* bt = block_tables + (int64_t)s * max_blocks;
  const int bs = 1 << bs_log2;
  const int64_t head_stride = (int64_t)bs * D;        // elements between heads in a block
  const int64_t block_stride = (int64_t)H * head_stride;

  float m = -INFINITY, l = 0.f;
  float acc[VEC];
#pragma unroll
  for (int j = 0; j < VEC; ++j) acc[j] = 0.f;

  for (int r0 = t_begin + warp * ROUND; r0 < t_end; r0 += PD_WARPS * ROUND) {
    Vec16<T> kv[U], vv[U];
    bool ok[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int t = r0 + u * TPW + grp;
      ok[u] = t < t_end;
      const int blk = ok[u] ? bt[t >> bs_log2] : 0;
      ok[u] = ok[u] && blk >= 0 && blk < num_blocks;  // bad ids read nothing
      if (ok[u]) {
        const int64_t off = blk * block_stride + h * head_stride +
                            (int64_t)(t & (bs - 1)) * D + dofs;
        kv[u] = ld_vec16_stream(k_cache + off);
        vv[u] = ld_vec16_stream(v_cache + off);
      }
    }
    float sc[U];
    float rmax = -INFINITY;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float d = 0.f;
      if (ok[u]) {
#pragma unroll
        for (int j = 0; j < VEC; ++j) d = fmaf(qf[j], to_f(kv[u].v[j]), d);
      }
#pragma unroll
      for (int off = LPT / 2; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
      sc[u] = ok[u] ? d : -INFINITY;
      rmax = fmaxf(rmax, sc[u]);
    }
#pragma unroll
    for (int off = 16; off >= LPT; off >>= 1)
      rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, off));
    // A round can be fully masked (bad block ids): keep the state unchanged then.
    const float m_new = fmaxf(m, rmax);
    const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
    const float alpha = exp2f(m - m_use);
    l *= alpha;
#pragma unroll
    for (int j = 0; j < VEC; ++j) acc[j] *= alpha;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const float p = exp2f(sc[u] - m_use);  // 0 for masked rows
      l += p;
      if (ok[u]) {
#pragma unroll
        for (int j = 0; j < VEC; ++j) acc[j] = fmaf(p, to_f(vv[u].v[j]), acc[j]);
      }
    }
    m = m_new;
  }

  // Merge token groups inside the warp (same d chunk, different rows).
#pragma unroll
  for (int off = 16; off >= LPT; off >>= 1) {
    l += __shfl_xor_sync(0xffffffffu, l, off);
#pragma unroll
    for (int j = 0; j < VEC; ++j) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], off);
  }

  __shared__ float sm_m[PD_WARPS], sm_l[PD_WARPS];
  __shared__ float sm_acc[PD_WARPS][D];
  if (lane == 0) { sm_m[warp] = m; sm_l[warp] = l; }
  if (grp == 0) {
#pragma unroll
    for (int j = 0; j < VEC; ++j) sm_acc[warp][dofs + j] = acc[j];
  }
  __syncthreads();

  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < PD_WARPS; ++w) M = fmaxf(M, sm_m[w]);
  float wts[PD_WARPS];
  float L = 0.f;
#pragma unroll
  for (int w = 0; w < PD_WARPS; ++w) {
    wts[w] = (sm_m[w] == -INFINITY) ? 0.f : exp2f(sm_m[w] - M);
    L += wts[w] * sm_l[w];
  }

  if (nparts <= 1) {
    T* orow = o + s * so_s + h * so_h;
    const float inv = L > 0.f ? 1.0f / L : 0.f;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      float a = 0.f;
#pragma unroll
      for (int w = 0; w < PD_WARPS; ++w) a = fmaf(wts[w], sm_acc[w][d], a);
      orow[d] = from_f<T>(a * inv);
    }
  } else {
    const int64_t pi = ((int64_t)s * H + h) * max_parts + part;
    if (threadIdx.x == 0) { part_m[pi] = M; part_l[pi] = L; }
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      float a = 0.f;
#pragma unroll
      for (int w = 0; w < PD_WARPS; ++w) a = fmaf(wts[w], sm_acc[w][d], a);
      part_acc[pi * D + d] = a;
    }
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(128)
paged_decode_combine_kernel(const int32_t* __restrict__ context_lens, int max_tokens,
                            T* __restrict__ o, int H, int64_t so_s, int64_t so_h, int max_parts,
                            const float* __restrict__ part_m, const float* __restrict__ part_l,
                            const float* __restrict__ part_acc) {
  allow_dependents();
  wait_prerequisites();
  const int h = blockIdx.x, s = blockIdx.y;
  const int ctx = max(0, min(context_lens[s], max_tokens));
  const int nparts = (ctx + PD_PART_TOKENS - 1) / PD_PART_TOKENS;
  if (nparts <= 1) return;  // written directly by the decode kernel
  const int64_t base = ((int64_t)s * H + h) * max_parts;
  float M = -INFINITY;
  for (int p = 0; p < nparts; ++p) M = fmaxf(M, part_m[base + p]);
  float L = 0.f;
  for (int p = 0; p < nparts; ++p) L += exp2f(part_m[base + p] - M) * part_l[base + p];
  const float inv = 1.0f / L;
  T* orow = o + s * so_s + h * so_h;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float a = 0.f;
    for (int p = 0; p < nparts; ++p)
      a = fmaf(exp2f(part_m[base + p] - M), part_acc[(base + p) * D + d], a);
    orow[d] = from_f<T>(a * inv);
  }
}

// Bulk-copy variant (block_size 16): one producer warp streams whole
// (block, head) runs of K and V -- BS*D contiguous elements each -- into a
// PD_STAGES-deep shared-memory ring with cp.async.bulk + mbarrier
// transaction counts, so every CTA keeps several KiB of HBM reads in flight
// with few registers; four consumer warps each score a quarter of each
// block's tokens from shared memory and keep the same online softmax as the
// register kernel above. Partial results use the same workspace layout.
constexpr int PD_STAGES = 4;
constexpr int PD_BS = 16;

template <typename T, int D>
__global__ void __launch_bounds__((PD_WARPS + 1) * 32)
paged_decode_bulk_kernel(const T* __restrict__ q, const T* __restrict__ k_cache,
                         const T* __restrict__ v_cache, const int32_t* __restrict__ block_tables,
                         const int32_t* __restrict__ context_lens, T* __restrict__ o, int H,
                         int max_blocks, int num_blocks, int64_t sq_s, int64_t sq_h, int64_t so_s,
                         int64_t so_h, float scale_log2, int max_parts, float* __restrict__ part_m,
                         float* __restrict__ part_l, float* __restrict__ part_acc) {
  allow_dependents();
  wait_prerequisites();
  using namespace sm100;
  constexpr int VEC = 16 / sizeof(T);
  constexpr int LPT = D / VEC;                    // lanes per token row
  constexpr int TPW = 32 / LPT;                   // token rows per warp-wide load
  constexpr int ROWS_PER_WARP = PD_BS / PD_WARPS; // rows of each block one warp scores
  constexpr int U = (ROWS_PER_WARP + TPW - 1) / TPW;
  constexpr int CH = PD_BS * D * (int)sizeof(T);  // bytes of one (block, head) run
  constexpr int BLK_PER_PART = PD_PART_TOKENS / PD_BS;
  static_assert(LPT >= 1 && LPT <= 32 && (32 % LPT) == 0, "unsupported head dim");
  static_assert(CH % 16 == 0, "bulk copies move multiples of 16 bytes");

  __shared__ __align__(128) uint8_t ring[PD_STAGES][2][CH];
  __shared__ __align__(8) uint64_t full[PD_STAGES], empty[PD_STAGES];
  __shared__ int valid[PD_STAGES];
  __shared__ float sm_m[PD_WARPS], sm_l[PD_WARPS];
  __shared__ float sm_acc[PD_WARPS][D];

  const int part = blockIdx.x, h = blockIdx.y, s = blockIdx.z;
  const int ctx = max(0, min(context_lens[s], max_blocks * PD_BS));
  const int t_begin = part * PD_PART_TOKENS;
  if (t_begin >= ctx && !(ctx == 0 && part == 0)) return;
  const int t_end = min(ctx, t_begin + PD_PART_TOKENS);
  const int nparts = (ctx + PD_PART_TOKENS - 1) / PD_PART_TOKENS;
  const int b0 = t_begin / PD_BS;
  const int nblk = (t_end - t_begin + PD_BS - 1) / PD_BS;
  (void)BLK_PER_PART;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < PD_STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], PD_WARPS);
    }
    fence_barrier_init();
  }
  __syncthreads();

  const int32_t* bt = block_tables + (int64_t)s * max_blocks;
  const int64_t head_off = (int64_t)h * PD_BS * D;
  const int64_t block_stride = (int64_t)H * PD_BS * D;

  float m = -INFINITY, l = 0.f;
  float acc[VEC];
#pragma unroll
  for (int j = 0; j < VEC; ++j) acc[j] = 0.f;
  const int grp = lane / LPT, dofs = (lane % LPT) * VEC;

  if (warp == PD_WARPS) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      for (int i = 0; i < nblk; ++i) {
        const int st = i % PD_STAGES;
        if (i >= PD_STAGES && !mbar_wait(&empty[st], ((i / PD_STAGES) - 1) & 1, 0x401)) break;
        const int blk = bt[b0 + i];
        if (blk >= 0 && blk < num_blocks) {
          valid[st] = 1;
          mbar_arrive_expect_tx(&full[st], 2 * CH);
          const int64_t off = blk * block_stride + head_off;
          bulk_load(ring[st][0], k_cache + off, CH, &full[st]);
          bulk_load(ring[st][1], v_cache + off, CH, &full[st]);
        } else {
          valid[st] = 0;  // a bad block id reads nothing; its tokens are masked
          mbar_arrive(&full[st]);
        }
      }
    }
  } else {
    // ----------------------------------------------------------- consumers --
    float qf[VEC];
    {
      Vec16<T> qv = ld_vec16(q + s * sq_s + h * sq_h + dofs);
#pragma unroll
      for (int j = 0; j < VEC; ++j) qf[j] = to_f(qv.v[j]) * scale_log2;
    }
    for (int i = 0; i < nblk; ++i) {
      const int st = i % PD_STAGES;
      if (!mbar_wait(&full[st], (i / PD_STAGES) & 1, 0x402)) break;
      const int tok0 = t_begin + i * PD_BS;
      const bool blk_ok = valid[st] != 0;
      float sc[U];
      Vec16<T> vv[U];
      float rmax = -INFINITY;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int r = warp * ROWS_PER_WARP + u * TPW + grp;
        const bool ok = blk_ok && (u * TPW + grp < ROWS_PER_WARP) && (tok0 + r < t_end);
        float d = 0.f;
        if (ok) {
          Vec16<T> kv = *reinterpret_cast<const Vec16<T>*>(ring[st][0] + (r * D + dofs) * sizeof(T));
          vv[u] = *reinterpret_cast<const Vec16<T>*>(ring[st][1] + (r * D + dofs) * sizeof(T));
#pragma unroll
          for (int j = 0; j < VEC; ++j) d = fmaf(qf[j], to_f(kv.v[j]), d);
        }
#pragma unroll
        for (int off = LPT / 2; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
        sc[u] = ok ? d : -INFINITY;
        rmax = fmaxf(rmax, sc[u]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
#pragma unroll
      for (int off = 16; off >= LPT; off >>= 1)
        rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, off));
      const float m_new = fmaxf(m, rmax);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      const float alpha = exp2f(m - m_use);
      l *= alpha;
#pragma unroll
      for (int j = 0; j < VEC; ++j) acc[j] *= alpha;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const float pw = exp2f(sc[u] - m_use);
        l += pw;
        if (sc[u] != -INFINITY) {
#pragma unroll
          for (int j = 0; j < VEC; ++j) acc[j] = fmaf(pw, to_f(vv[u].v[j]), acc[j]);
        }
      }
      m = m_new;
    }
#pragma unroll
    for (int off = 16; off >= LPT; off >>= 1) {
      l += __shfl_xor_sync(0xffffffffu, l, off);
#pragma unroll
      for (int j = 0; j < VEC; ++j) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], off);
    }
    if (lane == 0) { sm_m[warp] = m; sm_l[warp] = l; }
    if (grp == 0) {
#pragma unroll
      for (int j = 0; j < VEC; ++j) sm_acc[warp][dofs + j] = acc[j];
    }
  }
  __syncthreads();

  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < PD_WARPS; ++w) M = fmaxf(M, sm_m[w]);
  float wts[PD_WARPS];
  float L = 0.f;
#pragma unroll
  for (int w = 0; w < PD_WARPS; ++w) {
    wts[w] = (sm_m[w] == -INFINITY) ? 0.f : exp2f(sm_m[w] - M);
    L += wts[w] * sm_l[w];
  }
  if (nparts <= 1) {
    T* orow = o + s * so_s + h * so_h;
    const float inv = L > 0.f ? 1.0f / L : 0.f;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      float a = 0.f;
#pragma unroll
      for (int w = 0; w < PD_WARPS; ++w) a = fmaf(wts[w], sm_acc[w][d], a);
      orow[d] = from_f<T>(a * inv);
    }
  } else {
    const int64_t pi = ((int64_t)s * H + h) * max_parts + part;
    if (threadIdx.x == 0) { part_m[pi] = M; part_l[pi] = L; }
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      float a = 0.f;
#pragma unroll
      for (int w = 0; w < PD_WARPS; ++w) a = fmaf(wts[w], sm_acc[w][d], a);
      part_acc[pi * D + d] = a;
    }
  }
}

template <typename T, int D>
static int launch_paged_decode(const void* q, const void* kc, const void* vc,
                               const int32_t* bt, const int32_t* cl, void* o, int64_t S,
                               int64_t H, int64_t max_blocks, int64_t num_blocks, int bs_log2, int64_t sq_s,
                               int64_t sq_h, int64_t so_s, int64_t so_h, float scale,
                               void* ws, int64_t ws_bytes, cudaStream_t st) {
  const int64_t P = pd_max_parts(max_blocks, (int64_t)1 << bs_log2);
  float* pm = nullptr; float* pl = nullptr; float* pa = nullptr;
  if (P > 1) {
    const int64_t need = lsb_paged_decode_workspace_size(S, H, D, max_blocks, (int64_t)1 << bs_log2);
    LSB_CHECK_ARG(ws != nullptr && ws_bytes >= need,
                  "paged_decode: workspace of %lld bytes required, got %lld", (long long)need,
                  (long long)ws_bytes);
    LSB_CHECK_ARG(aligned16(ws), "paged_decode: workspace must be 16-byte aligned");
    pm = (float*)ws;
    pl = pm + S * H * P;
    pa = pl + S * H * P;
  }
  dim3 grid((unsigned)P, (unsigned)H, (unsigned)S);
  bool launched = false;
  if constexpr (PD_BS * D * sizeof(T) * 2 * PD_STAGES <= 40 * 1024) {
    if (bs_log2 == 4 && aligned16(kc) && aligned16(vc)) {
      LSB_CUDA_OK(launch_kernel(paged_decode_bulk_kernel<T, D>, grid, dim3((PD_WARPS + 1) * 32), 0,
                                st, (const T*)q, (const T*)kc, (const T*)vc, bt, cl, (T*)o, (int)H,
                                (int)max_blocks, (int)num_blocks, sq_s, sq_h, so_s, so_h,
                                scale * PD_LOG2E, (int)P, pm, pl, pa),
                  "paged_decode");
      launched = true;
    }
  }
  if (!launched)
  paged_decode_kernel<T, D><<<grid, PD_WARPS * 32, 0, st>>>(
      (const T*)q, (const T*)kc, (const T*)vc, bt, cl, (T*)o, (int)H, (int)max_blocks, (int)num_blocks, bs_log2,
      sq_s, sq_h, so_s, so_h, scale * PD_LOG2E, (int)P, pm, pl, pa);
  LSB_CHECK_LAUNCH("paged_decode");
  if (P > 1) {
    LSB_CUDA_OK(launch_kernel(paged_decode_combine_kernel<T, D>, dim3((unsigned)H, (unsigned)S),
                              dim3(128), 0, st, (const int32_t*)cl, (int)(max_blocks << bs_log2),
                              (T*)o, (int)H, so_s, so_h, (int)P, (const float*)pm,
                              (const float*)pl, (const float*)pa),
                "paged_decode_combine");
  }
  return LSB_OK;
}

template <typename T>
__global__ void kv_cache_write_kernel(const T* __restrict__ k, const T* __restrict__ v,
                                      T* __restrict__ k_cache, T* __restrict__ v_cache,
                                      const int64_t* __restrict__ slots, int64_t T_, int H, int D,
                                      int bs, int64_t num_blocks_x_bs, int64_t sk_t, int64_t sk_h, int64_t sv_t,
                                      int64_t sv_h, int vec) {
  // One warp per (token, head) row.
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= T_ * H) return;
  const int64_t t = row / H;
  const int h = (int)(row % H);
  const int64_t slot = slots[t];
  if (slot < 0 || slot >= (int64_t)num_blocks_x_bs) return;
  const int64_t blk = slot / bs, off = slot % bs;
  const int64_t dst = ((blk * H + h) * bs + off) * D;
  const T* ks = k + t * sk_t + h * sk_h;
  const T* vs = v + t * sv_t + h * sv_h;
  if (vec) {
    constexpr int VEC = 16 / sizeof(T);
    for (int d = lane * VEC; d < D; d += 32 * VEC) {
      st_vec16(k_cache + dst + d, ld_vec16(ks + d));
      st_vec16(v_cache + dst + d, ld_vec16(vs + d));
    }
  } else {
    for (int d = lane; d < D; d += 32) {
      k_cache[dst + d] = ks[d];
      v_cache[dst + d] = vs[d];
    }
  }
}

int paged_decode_device_error(bool reset) {
  return sm100::tu_device_error(reset);
}

}  // namespace lsb

extern "C" int64_t lsb_paged_decode_workspace_size(int64_t S, int64_t H, int64_t D,
                                                   int64_t max_blocks_per_seq,
                                                   int64_t block_size) {
  if (S <= 0 || H <= 0 || D <= 0 || max_blocks_per_seq <= 0 || block_size <= 0) return 0;
  const int64_t P = lsb::pd_max_parts(max_blocks_per_seq, block_size);
  if (P <= 1) return 0;
  return (int64_t)sizeof(float) * S * H * P * (D + 2);
}

extern "C" int lsb_paged_decode(const void* q, const void* k_cache, const void* v_cache,
                                const int32_t* block_tables, const int32_t* context_lens,
                                void* o, int64_t S, int64_t H, int64_t D,
                                int64_t max_blocks_per_seq, int64_t block_size,
                                int64_t num_blocks, int64_t sq_s, int64_t sq_h, int64_t so_s,
                                int64_t so_h, float scale, int dtype, void* workspace,
                                int64_t workspace_bytes, void* stream) {
  LSB_CHECK_ARG(S >= 0 && H > 0 && D > 0 && max_blocks_per_seq > 0 && num_blocks > 0,
                "paged_decode: bad sizes S=%lld H=%lld D=%lld max_blocks=%lld num_blocks=%lld",
                (long long)S, (long long)H, (long long)D, (long long)max_blocks_per_seq,
                (long long)num_blocks);
  LSB_CHECK_ARG(block_size > 0 && (block_size & (block_size - 1)) == 0,
                "paged_decode: block_size %lld must be a power of two", (long long)block_size);
  if (S == 0) return LSB_OK;
  LSB_CHECK_ARG(q && k_cache && v_cache && block_tables && context_lens && o,
                "paged_decode: null pointer");
  const int esz = lsb::dtype_size(dtype);
  LSB_CHECK_ARG(esz > 0, "paged_decode: unsupported dtype %d", dtype);
  LSB_CHECK_ARG(lsb::aligned16(q) && lsb::aligned16(k_cache) && lsb::aligned16(v_cache),
                "paged_decode: q and caches must be 16-byte aligned");
  LSB_CHECK_ARG((sq_s * esz) % 16 == 0 && (sq_h * esz) % 16 == 0,
                "paged_decode: q strides must be multiples of 16 bytes");
  LSB_CHECK_ARG(S <= 65535 && H <= 65535, "paged_decode: S or H above 65535");
  int bs_log2 = 0;
  while ((1LL << bs_log2) < block_size) ++bs_log2;
  cudaStream_t st = (cudaStream_t)stream;
  auto go = [&](auto tag, auto dtag) -> int {
    using T = decltype(tag);
    constexpr int DD = decltype(dtag)::value;
    return lsb::launch_paged_decode<T, DD>(q, k_cache, v_cache, block_tables, context_lens, o, S,
                                           H, max_blocks_per_seq, num_blocks, bs_log2, sq_s, sq_h, so_s, so_h,
                                           scale, workspace, workspace_bytes, st);
  };
  using I64 = std::integral_constant<int, 64>;
  using I128 = std::integral_constant<int, 128>;
  using I256 = std::integral_constant<int, 256>;
  using I32 = std::integral_constant<int, 32>;
  switch (dtype) {
    case LSB_DTYPE_BF16:
      if (D == 64) return go(__nv_bfloat16{}, I64{});
      if (D == 128) return go(__nv_bfloat16{}, I128{});
      if (D == 256) return go(__nv_bfloat16{}, I256{});
      break;
    case LSB_DTYPE_F16:
      if (D == 64) return go(__half{}, I64{});
      if (D == 128) return go(__half{}, I128{});
      if (D == 256) return go(__half{}, I256{});
      break;
    case LSB_DTYPE_F32:
      if (D == 32) return go(float{}, I32{});
      if (D == 64) return go(float{}, I64{});
      if (D == 128) return go(float{}, I128{});
      break;
  }
  lsb::set_error("paged_decode: head dim %lld unsupported for dtype %d", (long long)D, dtype);
  return LSB_ERR_UNSUPPORTED;
}

extern "C" int lsb_kv_cache_write(const void* k, const void* v, void* k_cache, void* v_cache,
                                  const int64_t* slot_mapping, int64_t T, int64_t H, int64_t D,
                                  int64_t num_blocks, int64_t block_size, int64_t sk_t,
                                  int64_t sk_h, int64_t sv_t, int64_t sv_h, int dtype,
                                  void* stream) {
  LSB_CHECK_ARG(T >= 0 && H > 0 && D > 0 && num_blocks > 0 && block_size > 0,
                "kv_cache_write: bad sizes");
  if (T == 0) return LSB_OK;
  LSB_CHECK_ARG(k && v && k_cache && v_cache && slot_mapping, "kv_cache_write: null pointer");
  const int esz = lsb::dtype_size(dtype);
  LSB_CHECK_ARG(esz > 0, "kv_cache_write: unsupported dtype %d", dtype);
  const bool vec = ((D * esz) % 16 == 0) && lsb::aligned16(k) && lsb::aligned16(v) &&
                   lsb::aligned16(k_cache) && lsb::aligned16(v_cache) &&
                   (sk_t * esz) % 16 == 0 && (sk_h * esz) % 16 == 0 && (sv_t * esz) % 16 == 0 &&
                   (sv_h * esz) % 16 == 0;
  const int64_t rows = T * H;
  const int threads = 256;
  const int64_t blocks = (rows * 32 + threads - 1) / threads;
  cudaStream_t st = (cudaStream_t)stream;
  return LSB_DISPATCH_DTYPE(dtype, Tt, [&] {
    lsb::kv_cache_write_kernel<Tt><<<(unsigned)blocks, threads, 0, st>>>(
        (const Tt*)k, (const Tt*)v, (Tt*)k_cache, (Tt*)v_cache, slot_mapping, T, (int)H, (int)D,
        (int)block_size, num_blocks * block_size, sk_t, sk_h, sv_t, sv_h, vec ? 1 : 0);
    LSB_CHECK_LAUNCH("kv_cache_write");
    return LSB_OK;
  });
}

// ---------------------------------------------------------------------------
// Allocation-free variant of lsb_paged_decode.
//
// Some callers cannot allocate device memory for the split-context scratch:
// runtimes that hand every byte of the GPU to their own memory pool (a
// cudaMalloc from a plugin would bypass their budget or fail under it), and
// thin FFI bindings (cgo, JNI, ctypes) that have no handle on the host
// framework's allocator. For them this entry point keeps the scratch in a
// fixed array inside the library instead of asking for a workspace.
//
// The array lives in every GPU that loads the library, until the process
// exits. Its host-side name is not a device address, so the device address is
// looked up once per device with cudaGetSymbolAddress (on that device's first
// call, which should therefore come before any stream capture) and passed to
// the kernels. Nothing in the array needs zeroing: every partial result the
// combine step reads is written by the same call first. All calls share the
// one array, so calls that overlap on the GPU (other streams, other threads)
// race and must be serialised by the caller.
namespace lsb {

constexpr int64_t kPdStaticScratchBytes = 8ll << 20;  // 8 MiB
static __device__ __align__(256) float g_pd_static_scratch[kPdStaticScratchBytes / 4];

static void* pd_static_scratch_ptr(int* rc) {
  static void* ptrs[64] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    set_error("paged_decode_static_scratch: cannot determine the current device");
    *rc = LSB_ERR_CUDA;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (ptrs[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_pd_static_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error("paged_decode_static_scratch: cudaGetSymbolAddress failed: %s",
                cudaGetErrorString(e));
      *rc = LSB_ERR_CUDA;
      return nullptr;
    }
    ptrs[dev] = p;
  }
  *rc = LSB_OK;
  return ptrs[dev];
}

}  // namespace lsb

extern "C" int64_t lsb_paged_decode_static_scratch_capacity(void) {
  return lsb::kPdStaticScratchBytes;
}

extern "C" int lsb_paged_decode_static_scratch(
    const void* q, const void* k_cache, const void* v_cache, const int32_t* block_tables,
    const int32_t* context_lens, void* o, int64_t S, int64_t H, int64_t D,
    int64_t max_blocks_per_seq, int64_t block_size, int64_t num_blocks, int64_t sq_s,
    int64_t sq_h, int64_t so_s, int64_t so_h, float scale, int dtype, void* stream) {
  const int64_t need =
      lsb_paged_decode_workspace_size(S, H, D, max_blocks_per_seq, block_size);
  LSB_CHECK_ARG(need <= lsb::kPdStaticScratchBytes,
                "paged_decode_static_scratch: these sizes need %lld bytes of scratch, above the "
                "built-in %lld-byte maximum; use lsb_paged_decode with a caller workspace",
                (long long)need, (long long)lsb::kPdStaticScratchBytes);
  void* ws = nullptr;
  if (need > 0) {
    int rc = LSB_OK;
    ws = lsb::pd_static_scratch_ptr(&rc);
    if (rc) return rc;
  }
  return lsb_paged_decode(q, k_cache, v_cache, block_tables, context_lens, o, S, H, D,
                          max_blocks_per_seq, block_size, num_blocks, sq_s, sq_h, so_s, so_h,
                          scale, dtype, ws, need, stream);
}

// ---------------------------------------------------------------------------
// Fused RoPE + paged KV-cache write for one decode step.
//
// Replaces, for the decode runner, the eager sequence of lightserve's
// apply_rope (model/minimal_llama.py:167-182: q*cos + rotate_half(q)*sin,
// each product and the sum rounded to the model dtype, as torch computes it)
// followed by the cache write, the block-table slot lookup
// (engine/block_manager.py:58-61) and the context-length update.
// Scalar form (any dtype, any alignment): one CTA per sequence, threads walk
// (head, rotation pair); 16-bit aligned inputs take the vectorised form below.
namespace lsb {

template <typename T>
__global__ void rope_kv_write_kernel(const T* __restrict__ qkv, int64_t s_s, int64_t s_part,
                                     int64_t s_h, const T* __restrict__ cos_t,
                                     const T* __restrict__ sin_t, int64_t s_pos,
                                     const int64_t* __restrict__ positions,
                                     const int32_t* __restrict__ block_tables, int max_blocks,
                                     T* __restrict__ q_out, T* __restrict__ k_cache,
                                     T* __restrict__ v_cache, int32_t* __restrict__ context_lens,
                                     int H, int D, int num_blocks, int bs) {
  const int s = blockIdx.x;
  const int64_t pos = positions[s];
  const int half = D / 2;
  const int64_t bidx = pos / bs;
  const int blk = (bidx >= 0 && bidx < max_blocks) ? block_tables[(int64_t)s * max_blocks + bidx] : -1;
  const bool write = blk >= 0 && blk < num_blocks;
  if (threadIdx.x == 0 && context_lens != nullptr) context_lens[s] = (int32_t)(pos + 1);
  const T* cs = cos_t + pos * s_pos;
  const T* sn = sin_t + pos * s_pos;
  const T* qrow = qkv + s * s_s;
  for (int idx = threadIdx.x; idx < H * half; idx += blockDim.x) {
    const int h = idx / half, i = idx % half;
    const float c0 = to_f(cs[i]), c1 = to_f(cs[i + half]);
    const float n0 = to_f(sn[i]), n1 = to_f(sn[i + half]);
    // rotate_half(x) = [-x2, x1]; every product and sum rounded to T.
    auto rope = [&](float x1, float x2, T& o1, T& o2) {
      const float a = to_f(from_f<T>(__fmul_rn(x1, c0)));
      const float b = to_f(from_f<T>(__fmul_rn(-x2, n0)));
      o1 = from_f<T>(__fadd_rn(a, b));
      const float c = to_f(from_f<T>(__fmul_rn(x2, c1)));
      const float d = to_f(from_f<T>(__fmul_rn(x1, n1)));
      o2 = from_f<T>(__fadd_rn(c, d));
    };
    const T* qh = qrow + h * s_h;
    const T* kh = qrow + s_part + h * s_h;
    const T* vh = qrow + 2 * s_part + h * s_h;
    T o1, o2;
    rope(to_f(qh[i]), to_f(qh[i + half]), o1, o2);
    T* qo = q_out + ((int64_t)s * H + h) * D;
    qo[i] = o1;
    qo[i + half] = o2;
    if (write) {
      const int64_t dst = (((int64_t)blk * H + h) * bs + (pos % bs)) * D;
      rope(to_f(kh[i]), to_f(kh[i + half]), o1, o2);
      k_cache[dst + i] = o1;
      k_cache[dst + i + half] = o2;
      v_cache[dst + i] = vh[i];
      v_cache[dst + i + half] = vh[i + half];
    }
  }
}

// Packed-prefill variant: one CTA per token of a [T, 3, H, D] QKV buffer,
// the token's cache slot given directly (slot_mapping, block * block_size +
// offset, < 0: no cache write, as in lsb_kv_cache_write). Rotated q and k
// also go to packed [T, H, D] outputs for the variable-length attention.
template <typename T>
__global__ void rope_kv_write_slots_kernel(const T* __restrict__ qkv, int64_t s_s, int64_t s_part,
                                           int64_t s_h, const T* __restrict__ cos_t,
                                           const T* __restrict__ sin_t, int64_t s_pos,
                                           const int64_t* __restrict__ positions,
                                           const int64_t* __restrict__ slot_mapping,
                                           T* __restrict__ q_out, T* __restrict__ k_out,
                                           T* __restrict__ k_cache, T* __restrict__ v_cache,
                                           int H, int D, int64_t num_slots, int bs) {
  const int64_t t = blockIdx.x;
  const int64_t pos = positions[t];
  const int64_t slot = slot_mapping[t];
  const bool write = slot >= 0 && slot < num_slots;
  const int64_t blk = slot / bs, off = slot % bs;
  const int half = D / 2;
  const T* cs = cos_t + pos * s_pos;
  const T* sn = sin_t + pos * s_pos;
  const T* row = qkv + t * s_s;
  for (int idx = threadIdx.x; idx < H * half; idx += blockDim.x) {
    const int h = idx / half, i = idx % half;
    const float c0 = to_f(cs[i]), c1 = to_f(cs[i + half]);
    const float n0 = to_f(sn[i]), n1 = to_f(sn[i + half]);
    // rotate_half(x) = [-x2, x1]; every product and sum rounded to T.
    auto rope = [&](float x1, float x2, T& o1, T& o2) {
      const float a = to_f(from_f<T>(__fmul_rn(x1, c0)));
      const float b = to_f(from_f<T>(__fmul_rn(-x2, n0)));
      o1 = from_f<T>(__fadd_rn(a, b));
      const float c = to_f(from_f<T>(__fmul_rn(x2, c1)));
      const float d = to_f(from_f<T>(__fmul_rn(x1, n1)));
      o2 = from_f<T>(__fadd_rn(c, d));
    };
    const T* qh = row + h * s_h;
    const T* kh = row + s_part + h * s_h;
    const T* vh = row + 2 * s_part + h * s_h;
    const int64_t o = (t * H + h) * D;
    T q1, q2, k1, k2;
    rope(to_f(qh[i]), to_f(qh[i + half]), q1, q2);
    rope(to_f(kh[i]), to_f(kh[i + half]), k1, k2);
    q_out[o + i] = q1;
    q_out[o + i + half] = q2;
    if (k_out != nullptr) {
      k_out[o + i] = k1;
      k_out[o + i + half] = k2;
    }
    if (write) {
      const int64_t dst = ((blk * H + h) * bs + off) * D;
      k_cache[dst + i] = k1;
      k_cache[dst + i + half] = k2;
      v_cache[dst + i] = vh[i];
      v_cache[dst + i + half] = vh[i + half];
    }
  }
}

// 16-byte vectorised forms for 16-bit types: a thread rotates 8 consecutive
// pairs (i, i + D/2) of one head of one token (16-byte loads of q, k, v, cos
// and sin, 16-byte stores); a 256-thread CTA covers 256 / (H * D / 16)
// tokens. Same roundings as the scalar kernels. The packed-prefill kernel
// takes each token's cache slot from slot_mapping, the decode kernel derives
// it from the sequence's block table and position (and sets its context
// length).
template <typename T>
__device__ __forceinline__ void rope_vec_lane(const T* __restrict__ qkv, int64_t s_s,
                                              int64_t s_part, int64_t s_h,
                                              const T* __restrict__ cos_t,
                                              const T* __restrict__ sin_t, int64_t s_pos,
                                              int64_t t, int h, int i0, int64_t pos, int64_t slot,
                                              T* __restrict__ q_out, T* __restrict__ k_out,
                                              T* __restrict__ k_cache, T* __restrict__ v_cache,
                                              int H, int D, int bs) {
  const int half = D / 2;
  const Vec16<T> c0 = ld_vec16(cos_t + pos * s_pos + i0), c1 = ld_vec16(cos_t + pos * s_pos + i0 + half);
  const Vec16<T> n0 = ld_vec16(sin_t + pos * s_pos + i0), n1 = ld_vec16(sin_t + pos * s_pos + i0 + half);
  const T* qh = qkv + t * s_s + h * s_h;
  const Vec16<T> q1 = ld_vec16(qh + i0), q2 = ld_vec16(qh + i0 + half);
  const Vec16<T> k1 = ld_vec16(qh + s_part + i0), k2 = ld_vec16(qh + s_part + i0 + half);
  Vec16<T> oq1, oq2, ok1, ok2;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float fc0 = to_f(c0.v[e]), fc1 = to_f(c1.v[e]), fn0 = to_f(n0.v[e]), fn1 = to_f(n1.v[e]);
    // rotate_half(x) = [-x2, x1]; every product and sum rounded to T.
    auto rope = [&](float x1, float x2, T& o1, T& o2) {
      const float a = to_f(from_f<T>(__fmul_rn(x1, fc0)));
      const float b = to_f(from_f<T>(__fmul_rn(-x2, fn0)));
      o1 = from_f<T>(__fadd_rn(a, b));
      const float c = to_f(from_f<T>(__fmul_rn(x2, fc1)));
      const float d = to_f(from_f<T>(__fmul_rn(x1, fn1)));
      o2 = from_f<T>(__fadd_rn(c, d));
    };
    rope(to_f(q1.v[e]), to_f(q2.v[e]), oq1.v[e], oq2.v[e]);
    rope(to_f(k1.v[e]), to_f(k2.v[e]), ok1.v[e], ok2.v[e]);
  }
  const int64_t o = (t * H + h) * D + i0;
  st_vec16(q_out + o, oq1);
  st_vec16(q_out + o + half, oq2);
  if (k_out != nullptr) {
    st_vec16(k_out + o, ok1);
    st_vec16(k_out + o + half, ok2);
  }
  if (slot >= 0) {
    const int64_t dst = (((slot / bs) * H + h) * bs + slot % bs) * D + i0;
    st_vec16(k_cache + dst, ok1);
    st_vec16(k_cache + dst + half, ok2);
    st_vec16(v_cache + dst, ld_vec16(qh + 2 * s_part + i0));
    st_vec16(v_cache + dst + half, ld_vec16(qh + 2 * s_part + i0 + half));
  }
}

template <typename T>
__global__ void __launch_bounds__(256)
rope_kv_write_slots_vec_kernel(const T* __restrict__ qkv, int64_t s_s, int64_t s_part, int64_t s_h,
                               const T* __restrict__ cos_t, const T* __restrict__ sin_t,
                               int64_t s_pos, const int64_t* __restrict__ positions,
                               const int64_t* __restrict__ slot_mapping, T* __restrict__ q_out,
                               T* __restrict__ k_out, T* __restrict__ k_cache,
                               T* __restrict__ v_cache, int H, int D, int64_t T_tokens,
                               int64_t num_slots, int bs) {
  const int half = D / 2;
  const int lanes_per_token = H * half / 8;
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t t = g / lanes_per_token;
  if (t >= T_tokens) return;
  const int r = (int)(g - t * lanes_per_token);
  const int h = r / (half / 8);
  const int i0 = (r - h * (half / 8)) * 8;
  const int64_t slot = slot_mapping[t];
  rope_vec_lane(qkv, s_s, s_part, s_h, cos_t, sin_t, s_pos, t, h, i0, positions[t],
                (slot >= 0 && slot < num_slots) ? slot : -1, q_out, k_out, k_cache, v_cache, H, D,
                bs);
}

template <typename T>
__global__ void __launch_bounds__(256)
rope_kv_write_vec_kernel(const T* __restrict__ qkv, int64_t s_s, int64_t s_part, int64_t s_h,
                         const T* __restrict__ cos_t, const T* __restrict__ sin_t, int64_t s_pos,
                         const int64_t* __restrict__ positions,
                         const int32_t* __restrict__ block_tables, int max_blocks,
                         T* __restrict__ q_out, T* __restrict__ k_cache, T* __restrict__ v_cache,
                         int32_t* __restrict__ context_lens, int H, int D, int64_t S,
                         int num_blocks, int bs) {
  allow_dependents();
  wait_prerequisites();
  const int half = D / 2;
  const int lanes_per_token = H * half / 8;
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t s = g / lanes_per_token;
  if (s >= S) return;
  const int r = (int)(g - s * lanes_per_token);
  const int h = r / (half / 8);
  const int i0 = (r - h * (half / 8)) * 8;
  const int64_t pos = positions[s];
  const int64_t bidx = pos / bs;
  const int blk = (bidx >= 0 && bidx < max_blocks) ? block_tables[s * max_blocks + bidx] : -1;
  const int64_t slot = (blk >= 0 && blk < num_blocks) ? (int64_t)blk * bs + pos % bs : -1;
  if (r == 0 && context_lens != nullptr) context_lens[s] = (int32_t)(pos + 1);
  rope_vec_lane(qkv, s_s, s_part, s_h, cos_t, sin_t, s_pos, s, h, i0, pos, slot, q_out,
                (T*)nullptr, k_cache, v_cache, H, D, bs);
}

}  // namespace lsb

extern "C" int lsb_rope_kv_write_slots(const void* qkv, int64_t s_s, int64_t s_part, int64_t s_h,
                                       const void* cos_table, const void* sin_table, int64_t s_pos,
                                       const int64_t* positions, const int64_t* slot_mapping,
                                       void* q_out, void* k_out, void* k_cache, void* v_cache,
                                       int64_t T, int64_t H, int64_t D, int64_t num_blocks,
                                       int64_t block_size, int dtype, void* stream) {
  LSB_CHECK_ARG(T >= 0 && H > 0 && D > 0 && (D % 2) == 0 && num_blocks > 0 && block_size > 0,
                "rope_kv_write_slots: bad sizes");
  if (T == 0) return LSB_OK;
  LSB_CHECK_ARG(qkv && cos_table && sin_table && positions && slot_mapping && q_out && k_cache &&
                    v_cache,
                "rope_kv_write_slots: null pointer");
  LSB_CHECK_ARG(T <= 0x7fffffff, "rope_kv_write_slots: T too large");
  cudaStream_t st = (cudaStream_t)stream;
  const bool a16 = [&] {
    auto al = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    return (D % 16) == 0 && al(qkv) && al(cos_table) && al(sin_table) && al(q_out) &&
           (k_out == nullptr || al(k_out)) && al(k_cache) && al(v_cache) && (s_s * 2) % 16 == 0 &&
           (s_part * 2) % 16 == 0 && (s_h * 2) % 16 == 0 && (s_pos * 2) % 16 == 0;
  }();
  if ((dtype == LSB_DTYPE_BF16 || dtype == LSB_DTYPE_F16) && a16) {
    const int64_t lanes = T * H * D / 16;
    const unsigned blocks = (unsigned)((lanes + 255) / 256);
    auto launch = [&](auto tag) -> int {
      using Tp = decltype(tag);
      lsb::rope_kv_write_slots_vec_kernel<Tp><<<blocks, 256, 0, st>>>(
          (const Tp*)qkv, s_s, s_part, s_h, (const Tp*)cos_table, (const Tp*)sin_table, s_pos,
          positions, slot_mapping, (Tp*)q_out, (Tp*)k_out, (Tp*)k_cache, (Tp*)v_cache, (int)H,
          (int)D, T, num_blocks * block_size, (int)block_size);
      LSB_CHECK_LAUNCH("rope_kv_write_slots");
      return LSB_OK;
    };
    return dtype == LSB_DTYPE_BF16 ? launch(__nv_bfloat16()) : launch(__half());
  }
  return LSB_DISPATCH_DTYPE(dtype, Tp, [&] {
    lsb::rope_kv_write_slots_kernel<Tp><<<(unsigned)T, 256, 0, st>>>(
        (const Tp*)qkv, s_s, s_part, s_h, (const Tp*)cos_table, (const Tp*)sin_table, s_pos,
        positions, slot_mapping, (Tp*)q_out, (Tp*)k_out, (Tp*)k_cache, (Tp*)v_cache, (int)H,
        (int)D, num_blocks * block_size, (int)block_size);
    LSB_CHECK_LAUNCH("rope_kv_write_slots");
    return LSB_OK;
  });
}

extern "C" int lsb_rope_kv_write(const void* qkv, int64_t s_s, int64_t s_part, int64_t s_h,
                                 const void* cos_table, const void* sin_table, int64_t s_pos,
                                 const int64_t* positions, const int32_t* block_tables,
                                 int64_t max_blocks_per_seq, void* q_out, void* k_cache,
                                 void* v_cache, int32_t* context_lens, int64_t S, int64_t H,
                                 int64_t D, int64_t num_blocks, int64_t block_size, int dtype,
                                 void* stream) {
  LSB_CHECK_ARG(S >= 0 && H > 0 && D > 0 && (D % 2) == 0 && num_blocks > 0 && block_size > 0 &&
                    max_blocks_per_seq > 0,
                "rope_kv_write: bad sizes");
  if (S == 0) return LSB_OK;
  LSB_CHECK_ARG(qkv && cos_table && sin_table && positions && block_tables && q_out && k_cache &&
                    v_cache,
                "rope_kv_write: null pointer");
  LSB_CHECK_ARG(S <= 0x7fffffff, "rope_kv_write: S too large");
  cudaStream_t st = (cudaStream_t)stream;
  const bool a16 = [&] {
    auto al = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    return (D % 16) == 0 && al(qkv) && al(cos_table) && al(sin_table) && al(q_out) &&
           al(k_cache) && al(v_cache) && (s_s * 2) % 16 == 0 && (s_part * 2) % 16 == 0 &&
           (s_h * 2) % 16 == 0 && (s_pos * 2) % 16 == 0;
  }();
  if ((dtype == LSB_DTYPE_BF16 || dtype == LSB_DTYPE_F16) && a16) {
    const int64_t lanes = S * H * D / 16;
    const unsigned blocks = (unsigned)((lanes + 255) / 256);
    auto launch = [&](auto tag) -> int {
      using Tp = decltype(tag);
      LSB_CUDA_OK(lsb::launch_kernel(
          lsb::rope_kv_write_vec_kernel<Tp>, dim3(blocks), dim3(256), 0, st, (const Tp*)qkv, s_s,
          s_part, s_h, (const Tp*)cos_table, (const Tp*)sin_table, s_pos, positions,
          block_tables, (int)max_blocks_per_seq, (Tp*)q_out, (Tp*)k_cache, (Tp*)v_cache,
          context_lens, (int)H, (int)D, S, (int)num_blocks, (int)block_size), "rope_kv_write");
      return LSB_OK;
    };
    return dtype == LSB_DTYPE_BF16 ? launch(__nv_bfloat16()) : launch(__half());
  }
  return LSB_DISPATCH_DTYPE(dtype, T, [&] {
    lsb::rope_kv_write_kernel<T><<<(unsigned)S, 256, 0, st>>>(
        (const T*)qkv, s_s, s_part, s_h, (const T*)cos_table, (const T*)sin_table, s_pos,
        positions, block_tables, (int)max_blocks_per_seq, (T*)q_out, (T*)k_cache, (T*)v_cache,
        context_lens, (int)H, (int)D, (int)num_blocks, (int)block_size);
    LSB_CHECK_LAUNCH("rope_kv_write");
    return LSB_OK;
  });
}
