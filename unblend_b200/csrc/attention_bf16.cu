// Persistent bf16 flash attention on the tcgen05 tensor cores (head dim 48 or 64).
//
// softmax(Q K^T * scale) V per (sequence, head) for BS-RoFormer's axial
// attention (unblend/roformer.py:478-511, 1135-1159) on the bf16 path. Q, K and
// V are bf16 in HBM (the QKV projection writes them, with the rotary rotation
// already applied), addressed like unblend_attention_tc2 through 5-D tensor
// maps (head span, row, inner batch, outer batch): every Q / K / V load is a box
// of 64 dims (one 128-byte swizzled row per key or query) starting at the
// head's first dim, so a 48-dim head's box also holds 16 dims of the next head
// (or zero fill past the last one), which no MMA reads: S = Q K^T runs
// HD / 16 K-steps and O = P V has N = HD.
//
// Work is a flat stream of (unit, key tile) pairs, a unit being 128 queries of
// one head of one sequence; each CTA walks its units in a grid-stride loop,
// so the loads, the QK^T of the next tile and the softmax of the current one
// overlap across unit boundaries (the 62-band sequences are one key tile
// each). Two CTAs share an SM.
//
//   warp 0     TMA producer: Q (double-buffered per unit), K/V tiles into a 3-stage ring
//   warp 1     MMA issue (one lane): S = Q K^T (kind::f16, SS) into a double-buffered
//              TMEM tile, then O += P V with P read from TMEM (TS) into the unit's
//              double-buffered O accumulator
//   warps 2-5  softmax, one query row per thread: scores from TMEM, running max with
//              lazy rescaling (O is rescaled in TMEM only when the max grows by more
//              than 2^8, so the stale-max exponentials stay <= 256), P packed as bf16
//              pairs over the first 32 columns of its S tile; at the unit end
//              O / l (times the gate) to global
//   warps 6-9  V tile transposed to V^T (keys contiguous, the K-major B operand of
//              P V) with ldmatrix.trans / stmatrix
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "tc_common.cuh"

namespace {

using namespace ub::tc;

constexpr int BQ = 128;
constexpr int BK = 64;
constexpr int BOX = 64;  // dims per load (128-byte rows)
constexpr int NT = 320;
constexpr int STAGES = 3;
constexpr int Q_BYTES = BQ * 128;  // 128 rows x 64 bf16
constexpr int T_BYTES = BK * 128;  // 64 rows x 64 bf16
constexpr int K_OFF = 0, V_OFF = T_BYTES, VT_OFF = 2 * T_BYTES;
constexpr int STAGE = 3 * T_BYTES;
constexpr int SMEM = 2 * Q_BYTES + STAGES * STAGE + 1024 + 256;
constexpr int S_COL = 0;     // two 64-column S / P tiles
constexpr int O_COL = 128;   // two 64-column O accumulators
constexpr int TMEM_COLS = 256;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units

struct Args {
  int heads, lq, lk, q_tiles, inner, nkv;
  int total_units;
  void* o;
  long long o_so, o_si, o_sr;
  int o_bf16;
  const float* gate;
  long long g_so, g_si, g_sr;
  float c;  // scale * log2(e)
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

struct Unit {
  int qt, h, bi, bo;
};

__device__ __forceinline__ Unit unit_of(const Args& a, int u) {
  Unit r;
  r.qt = u % a.q_tiles;
  r.h = (u / a.q_tiles) % a.heads;
  const int z = u / (a.q_tiles * a.heads);
  r.bi = z % a.inner;
  r.bo = z / a.inner;
  return r;
}

// V [64 keys x 64 dims] -> V^T [64 dims x 64 keys], both bf16 with 128-byte
// swizzled rows. Warp w (0..3) moves 16 of the 64 8x8 blocks.
__device__ __forceinline__ void transpose_v(uint32_t v, uint32_t vt, int w, int lane) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int blk = w * 16 + i * 4 + (lane >> 3);  // block handled by this lane's address
    const int kb = blk >> 3, db = blk & 7;
    const int r = lane & 7;
    const int key = kb * 8 + r;
    const uint32_t src = v + key * 128 + ((db ^ (key & 7)) << 4);
    uint32_t x0, x1, x2, x3;
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(x0), "=r"(x1), "=r"(x2), "=r"(x3)
                 : "r"(src));
    const int d = db * 8 + r;
    const uint32_t dst = vt + d * 128 + ((kb ^ (d & 7)) << 4);
    asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(x0), "r"(x1),
                 "r"(x2), "r"(x3)
                 : "memory");
  }
}

template <int HD>
__global__ void __launch_bounds__(NT, 2)
    attention_bf16_kernel(const __grid_constant__ CUtensorMap mapQ, const __grid_constant__ CUtensorMap mapK,
                          const __grid_constant__ CUtensorMap mapV, const __grid_constant__ Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;  // [2][Q_BYTES]
  uint8_t* sKV = smem + 2 * Q_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + STAGES * STAGE);
  uint64_t* q_full = bars;            // [2]
  uint64_t* q_free = q_full + 2;      // [2]
  uint64_t* kv_full = q_free + 2;     // [STAGES]
  uint64_t* kv_conv = kv_full + STAGES;
  uint64_t* kv_free = kv_conv + STAGES;
  uint64_t* s_full = kv_free + STAGES;  // [2]
  uint64_t* p_ready = s_full + 2;       // [2]
  uint64_t* o_done = p_ready + 2;       // [1]
  uint64_t* o_free = o_done + 1;        // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_free + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkv = a.nkv;
  // Units of this CTA and the length of its (unit, key tile) stream.
  const int my_units = blockIdx.x < a.total_units ? (a.total_units - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int n_total = my_units * nkv;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_free[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_ready[i], 4);
      mbar_init(&o_free[i], 4);
    }
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_conv[s], 4);
      mbar_init(&kv_free[s], 1);
    }
    mbar_init(o_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      bool ok = true;
      for (int gt = 0; gt < n_total && ok; ++gt) {
        const int i = gt / nkv, j = gt - (gt / nkv) * nkv;
        const Unit un = unit_of(a, blockIdx.x + i * gridDim.x);
        if (j == 0) {
          const int qb = i & 1;
          if (i >= 2 && !mbar_wait(&q_free[qb], ((i >> 1) - 1) & 1)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&q_full[qb], Q_BYTES);
          tma_load_4d(sQ + qb * Q_BYTES, &mapQ, &q_full[qb], un.h * HD, un.qt * BQ, un.bi, un.bo);
        }
        const int s = gt % STAGES, r = gt / STAGES;
        if (r > 0 && !mbar_wait(&kv_free[s], (r - 1) & 1)) {
          ok = false;
          break;
        }
        uint8_t* st = sKV + s * STAGE;
        mbar_expect_tx(&kv_full[s], 2 * T_BYTES);
        tma_load_4d(st + K_OFF, &mapK, &kv_full[s], un.h * HD, j * BK, un.bi, un.bo);
        tma_load_4d(st + V_OFF, &mapV, &kv_full[s], un.h * HD, j * BK, un.bi, un.bo);
      }
      if (!ok) atomicExch(&g_error_flag, 5);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc(1u, 64u);        // S = Q K^T: M = 128, N = 64 keys
      constexpr uint32_t idesc_pv = instr_desc(1u, (uint32_t)HD);  // O = P V: N = HD dims
      bool ok = true;
      auto issue_s = [&](int gt) -> bool {
        const int i = gt / nkv, j = gt - (gt / nkv) * nkv;
        const int s = gt % STAGES;
        if (j == 0 && !mbar_wait(&q_full[i & 1], (i >> 1) & 1)) return false;
        if (!mbar_wait(&kv_conv[s], (gt / STAGES) & 1)) return false;
        tc_fence_after();
        const uint32_t q = smem_u32(sQ + (i & 1) * Q_BYTES);
        const uint32_t k = smem_u32(sKV + s * STAGE + K_OFF);
        const uint32_t d = tmem + S_COL + (gt & 1) * 64;
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks)  // 16 head dims per MMA
          umma_bf16(d, smem_desc(q + 32 * ks, 128), smem_desc(k + 32 * ks, 128), idesc, ks > 0 ? 1u : 0u);
        umma_commit(&s_full[gt & 1]);
        if (j == nkv - 1) umma_commit(&q_free[i & 1]);
        return true;
      };
      if (n_total > 0) ok = issue_s(0);
      for (int gt = 0; gt < n_total && ok; ++gt) {
        if (gt + 1 < n_total && !issue_s(gt + 1)) {
          ok = false;
          break;
        }
        const int i = gt / nkv, j = gt - (gt / nkv) * nkv;
        const int ob = i & 1;
        if (j == 0 && i >= 2 && !mbar_wait(&o_free[ob], ((i >> 1) - 1) & 1)) {
          ok = false;
          break;
        }
        if (!mbar_wait(&p_ready[gt & 1], (gt >> 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int s = gt % STAGES;
        const uint32_t vt = smem_u32(sKV + s * STAGE + VT_OFF);
        const uint32_t p = tmem + S_COL + (gt & 1) * 64;
        const uint32_t o = tmem + O_COL + ob * 64;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)  // 16 keys per MMA: 8 TMEM columns of bf16 pairs
          umma_bf16_ts(o, p + 8 * ks, smem_desc(vt + 32 * ks, 128), idesc_pv, (j > 0 || ks > 0) ? 1u : 0u);
        umma_commit(&kv_free[s]);
        umma_commit(o_done);
      }
      if (!ok) atomicExch(&g_error_flag, 6);
    }
  } else if (warp >= 6) {
    const int w = warp - 6;
    for (int gt = 0; gt < n_total; ++gt) {
      const int s = gt % STAGES;
      if (!mbar_wait(&kv_full[s], (gt / STAGES) & 1)) break;
      uint8_t* st = sKV + s * STAGE;
      transpose_v(smem_u32(st + V_OFF), smem_u32(st + VT_OFF), w, lane);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&kv_conv[s]);
    }
  } else {
    // Softmax warps 2-5: thread = query row 32*(warp%4) + lane.
    const int qw = warp & 3;
    const int row = qw * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(qw * 32) << 16);
    float m_run = -INFINITY, l_run = 0.f;
    int od = 0;  // o_done completions consumed (one per P V product, in order)
    bool ok = true;
    for (int gt = 0; gt < n_total && ok; ++gt) {
      const int i = gt / nkv, j = gt - (gt / nkv) * nkv;
      const int ob = i & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[gt & 1], (gt >> 1) & 1))) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[64];
      {
        uint32_t (&s0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sv[0]);
        uint32_t (&s1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&sv[32]);
        tmem_ld32(lane_base + S_COL + (gt & 1) * 64, s0);
        tmem_ld32(lane_base + S_COL + (gt & 1) * 64 + 32, s1);
      }
      const int kbase = j * BK;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const float v = kbase + c < a.lk ? __uint_as_float(sv[c]) * a.c : -INFINITY;
        sv[c] = __float_as_uint(v);
        mx = fmaxf(mx, v);
      }
      float corr = 1.f;
      bool rescale = false;
      if (j == 0) {
        m_run = mx;
        l_run = 0.f;
      } else if (mx > m_run + RESCALE_THRESHOLD) {
        corr = ex2(m_run - mx);
        m_run = mx;
        rescale = true;
      }
      float sum = 0.f;
      uint32_t pk[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const float p0 = ex2(__uint_as_float(sv[2 * c]) - m_run);
        const float p1 = ex2(__uint_as_float(sv[2 * c + 1]) - m_run);
        sum += p0 + p1;
        __nv_bfloat162 b2 = __floats2bfloat162_rn(p0, p1);
        pk[c] = *reinterpret_cast<uint32_t*>(&b2);
      }
      l_run = l_run * corr + sum;
      // Every earlier P V product must be complete: P(gt) overwrites the S tile
      // that P(gt-2) occupied, and a rescale rewrites O.
      while (od < gt) {
        if (!__all_sync(0xffffffffu, mbar_wait(o_done, od & 1))) {
          ok = false;
          break;
        }
        ++od;
      }
      if (!ok) break;
      tc_fence_after();
      if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
          uint32_t oh[32];
          tmem_ld32(lane_base + O_COL + ob * 64 + 32 * half, oh);
#pragma unroll
          for (int c = 0; c < 32; ++c) oh[c] = __float_as_uint(__uint_as_float(oh[c]) * corr);
          tmem_st32(lane_base + O_COL + ob * 64 + 32 * half, oh);
        }
      }
      tmem_st32(lane_base + S_COL + (gt & 1) * 64, pk);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_ready[gt & 1]);

      if (j == nkv - 1) {
        // Unit complete: wait for its last P V, then O / l (x gate) to global.
        while (od < gt + 1) {
          if (!__all_sync(0xffffffffu, mbar_wait(o_done, od & 1))) {
            ok = false;
            break;
          }
          ++od;
        }
        if (!ok) break;
        tc_fence_after();
        uint32_t o0[32], o1[32];
        tmem_ld32(lane_base + O_COL + ob * 64, o0);
        tmem_ld32(lane_base + O_COL + ob * 64 + 32, o1);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&o_free[ob]);
        const Unit un = unit_of(a, blockIdx.x + i * gridDim.x);
        const int qrow = un.qt * BQ + row;
        if (qrow < a.lq) {
          float inv = 1.f / l_run;
          if (a.gate)
            inv *= __ldg(a.gate + (long long)un.bo * a.g_so + (long long)un.bi * a.g_si + (long long)qrow * a.g_sr +
                         un.h);
          const long long off = (long long)un.bo * a.o_so + (long long)un.bi * a.o_si + (long long)qrow * a.o_sr +
                                (long long)un.h * HD;
          if (a.o_bf16) {
            uint4* out = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.o) + off);
#pragma unroll
            for (int d8 = 0; d8 < HD / 8; ++d8) {
              uint32_t w4[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int d = d8 * 8 + 2 * e;
                const float v0 = __uint_as_float(d < 32 ? o0[d] : o1[d - 32]) * inv;
                const float v1 = __uint_as_float(d + 1 < 32 ? o0[d + 1] : o1[d - 31]) * inv;
                __nv_bfloat162 b2 = __floats2bfloat162_rn(v0, v1);
                w4[e] = *reinterpret_cast<uint32_t*>(&b2);
              }
              out[d8] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
            }
          } else {
            float4* out = reinterpret_cast<float4*>(reinterpret_cast<float*>(a.o) + off);
#pragma unroll
            for (int d4 = 0; d4 < HD / 4; ++d4) {
              const int d = d4 * 4;
              const uint32_t* src = d < 32 ? &o0[d] : &o1[d - 32];
              out[d4] = make_float4(__uint_as_float(src[0]) * inv, __uint_as_float(src[1]) * inv,
                                    __uint_as_float(src[2]) * inv, __uint_as_float(src[3]) * inv);
            }
          }
        }
      }
    }
    if (!ok) atomicExch(&g_error_flag, 7);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// (head span, row, inner, outer) map of one of Q / K / V: `span` = heads * hd dims per row.
bool head_map(CUtensorMap* m, const void* base, int span, int rows, int inner, int outer, long long row_stride,
              long long inner_stride, long long outer_stride, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[4] = {(cuuint64_t)span, (cuuint64_t)rows, (cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[3] = {(cuuint64_t)row_stride * 2, (cuuint64_t)inner_stride * 2, (cuuint64_t)outer_stride * 2};
  cuuint32_t box[4] = {BOX, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

long long legal_stride(long long s, int extent) { return extent == 1 && s <= 0 ? 8 : s; }

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ub::kNumSMs;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return ub::kNumSMs;
  return n;
}

}  // namespace

extern "C" int unblend_attention_bf16(const void* q, const void* k, const void* v, const UnblendAttnParams* p,
                                      void* stream) {
  UB_REQUIRE(q && k && v && p && p->out);
  UB_REQUIRE(p->outer > 0 && p->inner > 0 && p->heads > 0 && p->lq > 0 && p->lk > 0 && (p->hd == 48 || p->hd == 64));
  UB_REQUIRE(p->rope == nullptr);  // rotary is applied by the producer of Q and K on this path
  const long long q_so = legal_stride(p->q_so, p->outer), q_si = legal_stride(p->q_si, p->inner);
  const long long kv_so = legal_stride(p->kv_so, p->outer), kv_si = legal_stride(p->kv_si, p->inner);
  UB_REQUIRE(p->q_sr > 0 && p->kv_sr > 0 && q_so > 0 && q_si > 0 && kv_so > 0 && kv_si > 0);
  UB_REQUIRE(p->q_sr % 8 == 0 && q_so % 8 == 0 && q_si % 8 == 0 && p->kv_sr % 8 == 0 && kv_so % 8 == 0 &&
             kv_si % 8 == 0);
  UB_REQUIRE(p->o_sr % 8 == 0 && p->o_so % 8 == 0 && p->o_si % 8 == 0);
  UB_REQUIRE((reinterpret_cast<uintptr_t>(q) & 15) == 0 && (reinterpret_cast<uintptr_t>(k) & 15) == 0 &&
             (reinterpret_cast<uintptr_t>(v) & 15) == 0 && (reinterpret_cast<uintptr_t>(p->out) & 15) == 0);
  // Row strides must cover the head span (the tensor maps bound each row to it).
  const int span = p->heads * p->hd;
  UB_REQUIRE(p->q_sr >= span && p->kv_sr >= span && p->o_sr >= span);
  CUtensorMap mq, mk, mv;
  if (!head_map(&mq, q, span, p->lq, p->inner, p->outer, p->q_sr, q_si, q_so, BQ) ||
      !head_map(&mk, k, span, p->lk, p->inner, p->outer, p->kv_sr, kv_si, kv_so, BK) ||
      !head_map(&mv, v, span, p->lk, p->inner, p->outer, p->kv_sr, kv_si, kv_so, BK))
    return UNBLEND_ERR_INVALID;
  Args a{};
  a.heads = p->heads;
  a.lq = p->lq;
  a.lk = p->lk;
  a.q_tiles = (p->lq + BQ - 1) / BQ;
  a.inner = p->inner;
  a.nkv = (p->lk + BK - 1) / BK;
  const long long units = (long long)p->outer * p->inner * p->heads * a.q_tiles;
  UB_REQUIRE(units < (1LL << 31) && units * a.nkv < (1LL << 31));
  a.total_units = (int)units;
  a.o = p->out;
  a.o_so = p->o_so;
  a.o_si = p->o_si;
  a.o_sr = p->o_sr;
  a.o_bf16 = p->out_bf16 ? 1 : 0;
  a.gate = p->gate;
  a.g_so = p->g_so;
  a.g_si = p->g_si;
  a.g_sr = p->g_sr;
  a.c = p->scale * 1.4426950408889634f;
  auto kern = p->hd == 48 ? attention_bf16_kernel<48> : attention_bf16_kernel<64>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
  // Persistent, two CTAs per SM (96 registers x 320 threads and ~105 KB of
  // shared memory each). The occupancy query answers 1 here, but two co-resident
  // CTAs were measured 1.4x faster on the 801-frame RoFormer sequences.
  long long grid = 2LL * sm_count();
  if (grid > units) grid = units;
  kern<<<(unsigned)grid, NT, SMEM, ub::as_stream(stream)>>>(mq, mk, mv, a);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_attention_bf16_error_flag(int* out_host, int clear) {
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
