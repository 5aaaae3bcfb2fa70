// Bidirectional LSTM recurrence of SCNet's DualPathRNN (unblend/scnet.py:440-500) on the
// tcgen05 tensor cores, for the bf16 precision setting (hidden 128 or 256).
//
// Per step and direction the gates of G = 64 sequences are
//   pre = xp[seq, step] + W_hh h_prev[seq]   (xp: both directions' input projections, fp32)
// A thread-block cluster of Q = hid / 32 CTAs owns one direction of 64 sequences; CTA r
// owns hidden units [32 r, 32 r + 32). Its 128 gate rows of W_hh (gate-major: row
// 32 q + u is gate q of unit 32 r + u) stay in shared memory as bf16 for the whole launch
// (the A operand, K-major, 128-byte swizzle), and every CTA keeps h_prev of the 64
// sequences as bf16 (the B operand, [seq][unit], double-buffered). One elected thread
// issues hid / 16 kind::f16 MMAs (M = 128 gate rows, N = 64 sequences) into TMEM; the eight
// warps (warp w reads gate w % 4, its TMEM lane quarter, for 32 of the sequences) move the
// gates to shared memory as [seq][gate][unit]; thread (unit u, 8 sequences) adds the input projections
// (prefetched into shared memory by cp.async during the previous step), applies the
// sigmoid / tanh cell update with the fp32 cell state in registers, stores h (fp32) and
// writes its bf16 copy; the CTA's 64 x 32 block of new h then goes to the B buffer of every
// CTA of the cluster through distributed shared memory, and one cluster barrier per step
// publishes it. W_hh and h are rounded to bf16 (the cell state, the gate sums and the
// input projections stay fp32).
#include <cuda_bf16.h>

#include "common.cuh"
#include "tc_common.cuh"

namespace {

using namespace ub::tc;

constexpr int LT_G = 64;    // sequences per cluster (MMA N)
constexpr int LT_NT = 256;  // threads per CTA: two per TMEM lane / gate row (one per column half)
constexpr int LT_DS = 129;  // row stride (floats) of the gate staging [seq][4 x 32]

template <int HID>
struct LtLayout {
  static constexpr int KCH = HID / 64;                  // 64-wide K chunks (128-byte rows)
  static constexpr int A_BYTES = KCH * 128 * 128;       // W slice: KCH x [128 rows x 128 B]
  static constexpr int B_BYTES = KCH * LT_G * 128;      // h: KCH x [64 rows x 128 B], one buffer
  static constexpr int A_OFF = 0;
  static constexpr int B_OFF = A_BYTES;                 // two B buffers
  static constexpr int D_OFF = B_OFF + 2 * B_BYTES;     // gates [64][129] fp32
  static constexpr int X_OFF = D_OFF + ((LT_G * LT_DS * 4 + 1023) / 1024) * 1024;  // xp [64][4][32] fp32
  static constexpr int H_OFF = X_OFF + LT_G * 128 * 4;  // new h, bf16 [64][32]
  static constexpr int BAR_OFF = H_OFF + LT_G * 32 * 2;
  static constexpr int SMEM = BAR_OFF + 64 + 1024;      // barriers, TMEM slot, alignment slack
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

// Byte offset of element (row, k) of a K-major bf16 operand stored as 64-wide K chunks of
// `rows` x 128-byte rows with the 128-byte swizzle (16-byte unit index XOR row % 8).
__device__ __forceinline__ uint32_t sw_off(int row, int k, int rows) {
  const int kc = k >> 6, kk = k & 63;
  return (uint32_t)(kc * rows * 128 + row * 128 + ((((kk >> 3) ^ (row & 7))) << 4) + (kk & 7) * 2);
}

__device__ __forceinline__ uint32_t lt_cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void lt_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void lt_st_remote(uint32_t local_addr, uint32_t rank, uint4 v) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
  asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(remote), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

// Fast sigmoid and tanh from the hardware exponential and an approximate division
// (~1e-7 absolute error; the bf16 recurrence rounds h to 2^-9 anyway).
__device__ __forceinline__ float lt_sigmoid(float v) { return __fdividef(1.0f, 1.0f + __expf(-v)); }
__device__ __forceinline__ float lt_tanh(float v) { return 1.0f - __fdividef(2.0f, 1.0f + __expf(2.0f * v)); }

template <int HID>
__global__ void __launch_bounds__(LT_NT, 1)
    lstm_tc_kernel(const float* __restrict__ xp, const float* __restrict__ whh_t, float* __restrict__ h_out,
                   int n_seq, int steps, int inner, long long outer_stride, long long inner_stride,
                   long long step_stride) {
  using L = LtLayout<HID>;
  constexpr int Q = HID / 32;
  extern __shared__ uint8_t lt_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(lt_raw) + 1023) & ~uintptr_t(1023));
  float* d_s = reinterpret_cast<float*>(smem + L::D_OFF);
  float* x_s = reinterpret_cast<float*>(smem + L::X_OFF);
  __nv_bfloat16* h_s = reinterpret_cast<__nv_bfloat16*>(smem + L::H_OFF);
  uint64_t* mma_done = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::BAR_OFF + 8);
  __shared__ long long rowb[LT_G];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t rank = lt_cluster_rank();
  const int dir = blockIdx.y;
  const int s0 = (blockIdx.x / Q) * LT_G;  // first sequence of the cluster
  const float* w = whh_t + (long long)dir * HID * 4 * HID;

  // W_hh rows of this CTA (gate-major: row 32 q + u = gate q of unit 32 rank + u) as bf16.
  for (int i = tid; i < 128 * HID; i += LT_NT) {
    const int k = i >> 7, row = i & 127;
    const float v = __ldg(w + (long long)k * 4 * HID + (row >> 5) * HID + 32 * (int)rank + (row & 31));
    *reinterpret_cast<__nv_bfloat16*>(smem + L::A_OFF + sw_off(row, k, 128)) = __float2bfloat16_rn(v);
  }
  // h_prev = 0 for the first step (buffer 0).
  for (int i = tid; i < L::B_BYTES / 16; i += LT_NT)
    reinterpret_cast<uint4*>(smem + L::B_OFF)[i] = make_uint4(0u, 0u, 0u, 0u);
  if (tid < LT_G) {
    const int s = s0 + tid < n_seq ? s0 + tid : 0;
    rowb[tid] = (long long)(s / inner) * outer_stride + (long long)(s % inner) * inner_stride;
  }
  if (tid == 0) {
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, 64);
  __syncthreads();

  // Input projections of a step -> x_s [seq][gate][unit] (16-byte cp.async, 16 per thread).
  const int n_live = n_seq - s0 < LT_G ? n_seq - s0 : LT_G;
  auto prefetch_xp = [&](int step) {
#pragma unroll 4
    for (int j = 0; j < LT_G * 4 * 8 / LT_NT; ++j) {
      const int i = tid + LT_NT * j;
      const int s = i >> 5, q = (i >> 3) & 3, u4 = i & 7;
      if (s < n_live) {
        const float* src = xp + (rowb[s] + step * step_stride) * (8LL * HID) + dir * 4LL * HID + q * HID +
                           32 * (int)rank + 4 * u4;
        cp_async16(smem_u32(x_s + s * 128 + q * 32 + 4 * u4), src);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  prefetch_xp(dir == 0 ? 0 : steps - 1);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  tc_fence_before();
  lt_cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  constexpr uint32_t idesc = instr_desc(1u, (uint32_t)LT_G);
  float cst[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) cst[j] = 0.f;
  bool ok = true;

  for (int it = 0; it < steps; ++it) {
    const int step = dir == 0 ? it : steps - 1 - it;
    const uint32_t bcur = smem_u32(smem + L::B_OFF + (it & 1) * L::B_BYTES);
    if (tid == 0) {
      const uint32_t a0 = smem_u32(smem + L::A_OFF);
#pragma unroll
      for (int ks = 0; ks < HID / 16; ++ks) {
        const uint32_t ko = (uint32_t)((ks & 3) * 32);  // 16 bf16 (32 bytes) per K step along the row
        const uint64_t da = smem_desc(a0 + (ks >> 2) * (128 * 128) + ko, 128);
        const uint64_t db = smem_desc(bcur + (ks >> 2) * (LT_G * 128) + ko, 128);
        umma_bf16(tmem, da, db, idesc, ks > 0 ? 1u : 0u);
      }
      umma_commit(mma_done);
    }
    ok = mbar_wait(mma_done, it & 1) && ok;
    tc_fence_after();
    // Gates of this warp's TMEM lane quarter (gate q = warp % 4), sequences 32 (warp / 4) ..
    // + 31 -> d_s[seq][q * 32 + unit].
    {
      const int q = warp & 3, half = warp >> 2;
      uint32_t v[32];
      tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + 32 * half, v);
#pragma unroll
      for (int j = 0; j < 32; ++j) d_s[(32 * half + j) * LT_DS + q * 32 + lane] = __uint_as_float(v[j]);
    }
    tc_fence_before();
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    // Cell update of unit `lane` for sequences 8 warp .. 8 warp + 7.
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int s = 8 * warp + j;
      const float* ds = d_s + s * LT_DS + lane;
      const float* xs = x_s + s * 128 + lane;
      const float ig = lt_sigmoid(ds[0] + xs[0]);
      const float fg = lt_sigmoid(ds[32] + xs[32]);
      const float gg = lt_tanh(ds[64] + xs[64]);
      const float og = lt_sigmoid(ds[96] + xs[96]);
      cst[j] = fg * cst[j] + ig * gg;
      const float hv = og * lt_tanh(cst[j]);
      if (s < n_live)
        h_out[(rowb[s] + step * step_stride) * (2LL * HID) + dir * (long long)HID + 32 * (int)rank + lane] = hv;
      h_s[s * 32 + lane] = __float2bfloat16_rn(hv);
    }
    __syncthreads();
    if (it + 1 < steps) prefetch_xp(dir == 0 ? it + 1 : steps - 2 - it);
    // The CTA's 64 x 32 block of new h into the next B buffer of every CTA of the cluster.
    const uint32_t bnext = smem_u32(smem + L::B_OFF + ((it + 1) & 1) * L::B_BYTES);
    {
      const int chunk = tid;  // 256 chunks of 8 units: (sequence, unit octet)
      const int s = chunk >> 2, i = chunk & 3;
      const uint4 v = *reinterpret_cast<const uint4*>(h_s + s * 32 + 8 * i);
      const uint32_t dst = bnext + sw_off(s, 32 * (int)rank + 8 * i, LT_G);
#pragma unroll
      for (int r = 0; r < Q; ++r) lt_st_remote(dst, (uint32_t)r, v);
    }
    asm volatile("fence.proxy.async.shared::cluster;" ::: "memory");
    tc_fence_before();
    lt_cluster_sync();
    tc_fence_after();
  }
  if (!ok && tid == 0) atomicExch(&g_error_flag, 4);
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 64);
  }
}

template <int HID>
cudaError_t launch_lstm_tc(const float* xp, const float* whh_t, float* h_out, int n_seq, int steps, int inner,
                           long long outer_stride, long long inner_stride, long long step_stride, cudaStream_t st) {
  using L = LtLayout<HID>;
  constexpr int Q = HID / 32;
  cudaError_t e =
      cudaFuncSetAttribute(lstm_tc_kernel<HID>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((n_seq + LT_G - 1) / LT_G) * Q, 2, 1);
  cfg.blockDim = dim3(LT_NT, 1, 1);
  cfg.dynamicSmemBytes = L::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = Q;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, lstm_tc_kernel<HID>, xp, whh_t, h_out, n_seq, steps, inner, outer_stride,
                            inner_stride, step_stride);
}

}  // namespace

// The recurrence with W_hh and h in bf16 on the tensor cores (hidden 128 or 256; other
// sizes return UNBLEND_ERR_INVALID and take unblend_lstm_recurrence).
extern "C" int unblend_lstm_recurrence_bf16(const float* xp, const float* whh_t, float* h_out, int n_seq, int steps,
                                            int hid, int inner, long long outer_stride, long long inner_stride,
                                            long long step_stride, void* stream) {
  UB_REQUIRE(xp && whh_t && h_out && n_seq > 0 && steps > 0 && inner > 0);
  UB_REQUIRE(hid == 128 || hid == 256);
  UB_REQUIRE((reinterpret_cast<uintptr_t>(xp) & 15) == 0);
  cudaStream_t st = ub::as_stream(stream);
  const cudaError_t e = hid == 128 ? launch_lstm_tc<128>(xp, whh_t, h_out, n_seq, steps, inner, outer_stride,
                                                         inner_stride, step_stride, st)
                                   : launch_lstm_tc<256>(xp, whh_t, h_out, n_seq, steps, inner, outer_stride,
                                                         inner_stride, step_stride, st);
  if (e != cudaSuccess) return (int)e;
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_lstm_error_flag(int* out_host, int clear) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_error_flag, sizeof(int));
  if (e != cudaSuccess) return (int)e;
  if (out_host) *out_host = v;
  if (clear) {
    int z = 0;
    e = cudaMemcpyToSymbol(g_error_flag, &z, sizeof(int));
    if (e != cudaSuccess) return (int)e;
  }
  return 0;
}
