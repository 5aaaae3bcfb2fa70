// Flash attention on the tcgen05 tensor cores.
//
// softmax(Q K^T * scale) V per (batch, head), as nn.MultiheadAttention
// computes it in eval mode without masks (unblend/transformer.py:290-301
// self-attention, 402-412 cross-attention), streaming K/V in tiles of 64 keys
// with an online softmax. One CTA owns 128 queries of one head (head dim <= 64).
//
//   warp 0     TMA producer: Q once, then K/V tiles into a 2-3 stage ring
//   warp 1     MMA issue: S = Q K^T into TMEM, then O += P V with P read from
//              TMEM (the A operand) and V^T from shared memory (K-major B)
//   warps 2-5  softmax: one query row per thread; read S from TMEM, update
//              the running max / sum, write P back over S in TMEM, rescale the
//              O row in TMEM only when its max moved; final O / l to global
//   warps 6-9  operand preparation: TF32 rounding / hi-lo split of Q and K in
//              place, and V transposed to V^T (keys contiguous) while split
// MODE 0 (fp32 accuracy): every product is hi*hi + hi*lo + lo*hi in
// kind::tf32 (3 MMAs). MODE 1: single-pass TF32 with round-to-nearest
// operands (used by the bf16 precision setting). MODE 2 (fp32 accuracy): the
// same three products with bf16 hi / lo parts (hi = x rounded to bf16, lo =
// x - hi rounded to bf16) in kind::f16, 16 dims or keys per MMA instead of 8:
// Q, K and V^T become bf16 hi / lo tiles (128-byte rows, 128-byte swizzle)
// beside their fp32 staging, and P is packed as bf16 hi / lo pairs over its S tile.
// MODE 2 runs two query tiles per CTA (attention_tc_pair_kernel below), whose
// softmax chains overlap on the tensor pipe.
// Q is multiplied by scale * log2(e) while it is split, so scores arrive in log2 units.
//
// Sequences are indexed by a two-level batch (outer, inner) with independent
// strides, so BS-RoFormer's axial attention reads its [batch, frames, bands,
// dim] tokens in place: along frames with (outer, inner) = (batch, band) and
// along bands with (batch * frame, 1) (unblend/roformer.py:1135-1159).
// Optional fusions for BS-RoFormer's gated rotary attention
// (unblend/roformer.py:478-511): the rotary rotation of Q and K at their
// sequence positions (interleaved pairs, unblend/roformer.py:251-271) is
// applied by the operand-preparation warps before rounding, and the output is
// multiplied by a per-(token, head) gate.
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "tc_common.cuh"

namespace {

using namespace ub::tc;

constexpr int BQ = 128;
constexpr int BK = 64;
constexpr int NT = 320;

// Layout of the one-query-tile kernel (MODE 0 and 1; MODE 2 runs attention_tc_pair_kernel).
template <int MODE>
struct AL {
  static_assert(MODE == 0 || MODE == 1, "TF32 modes");
  static constexpr int Q_BYTES = 2 * BQ * 128;   // 2 boxes of 32 dims x 128 rows (fp32)
  static constexpr int KV_BYTES = 2 * BK * 128;  // 2 boxes of 32 dims x 64 keys, or V^T (64 dims x 64 keys)
  static constexpr int Q_TOTAL = MODE == 0 ? 2 * Q_BYTES : Q_BYTES;  // hi in place [+ lo]
  // Stage: K (hi in place) [, K lo], V staging, V^T hi [, V^T lo].
  static constexpr int K_OFF = 0;
  static constexpr int KLO_OFF = KV_BYTES;
  static constexpr int V_OFF = MODE == 0 ? 2 * KV_BYTES : KV_BYTES;
  static constexpr int VT_OFF = V_OFF + KV_BYTES;
  static constexpr int VTLO_OFF = VT_OFF + KV_BYTES;
  static constexpr int STAGE = MODE == 0 ? VTLO_OFF + KV_BYTES : VT_OFF + KV_BYTES;
  static constexpr int STAGES = MODE == 0 ? 2 : 3;
  static constexpr int SMEM = Q_TOTAL + STAGES * STAGE + 1024 + 256;
  // TMEM columns: S/P double buffer, P lo double buffer (MODE 0), and the P V
  // product of the current tile.
  static constexpr int S_COL = 0;
  static constexpr int PLO_COL = 128;
  static constexpr int O_COL = MODE == 0 ? 256 : 128;
  static constexpr int TMEM_COLS = MODE == 0 ? 512 : 256;
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

struct AttnArgs {
  int heads, lq, lk, hd;
  int q_tiles, inner;
  void* o;
  long long o_so, o_si, o_sr;
  int o_bf16;
  const float* gate;
  long long g_so, g_si, g_sr;
  const float2* rope;  // [rope_len, hd/2] (cos, sin) or null
  int rope_len;
  float c;  // scale * log2(e)
};

__device__ __forceinline__ float tf32_round(float v) {
  return __uint_as_float((__float_as_uint(v) + 0x1000u) & 0xFFFFE000u);
}

// Byte offset of element (row r, column c < 32) of a [rows x 32] fp32 tile
// stored with 128-byte rows and the 128-byte swizzle.
__device__ __forceinline__ int sw128(int r, int c) { return r * 128 + ((((c >> 2) ^ (r & 7))) << 4) + (c & 3) * 4; }

// Round `n4` float4s at p to TF32 in place; with MODE 0 also write the residuals at lo.
// The tile is 2 boxes of [box_rows x 32 dims] (128-byte swizzled rows) whose
// row r holds sequence position pos0 + r; with `rope`, each (even, odd) dim
// pair is first rotated by the (cos, sin) of that position; every value is then
// multiplied by `mul` (the softmax scale times log2(e) for Q, 1 for K).
template <int MODE>
__device__ __forceinline__ void split_tile(uint8_t* p, uint8_t* lo, int n4, int t, int nt, int box_rows, int pos0,
                                           const float2* __restrict__ rope, int rope_len, int hd, float mul) {
  float4* h = reinterpret_cast<float4*>(p);
  float4* l = reinterpret_cast<float4*>(lo);
  for (int i = t; i < n4; i += nt) {
    float4 v = h[i];
    if (rope) {
      const int box = i / (box_rows * 8), within = i - box * (box_rows * 8);
      const int row = within >> 3;
      const int d0 = box * 32 + (((within & 7) ^ (row & 7)) << 2);
      if (d0 < hd) {
        int pos = pos0 + row;
        pos = pos < rope_len ? pos : rope_len - 1;
        const float2 cs0 = __ldg(rope + (long long)pos * (hd >> 1) + (d0 >> 1));
        const float2 cs1 = __ldg(rope + (long long)pos * (hd >> 1) + (d0 >> 1) + 1);
        v = make_float4(v.x * cs0.x - v.y * cs0.y, v.x * cs0.y + v.y * cs0.x, v.z * cs1.x - v.w * cs1.y,
                        v.z * cs1.y + v.w * cs1.x);
      }
    }
    v = make_float4(v.x * mul, v.y * mul, v.z * mul, v.w * mul);
    float4 vh;
    vh.x = tf32_round(v.x);
    vh.y = tf32_round(v.y);
    vh.z = tf32_round(v.z);
    vh.w = tf32_round(v.w);
    h[i] = vh;
    if (MODE == 0) l[i] = make_float4(v.x - vh.x, v.y - vh.y, v.z - vh.z, v.w - vh.w);
  }
}

// V staging [2 boxes of (64 keys x 32 dims)] -> V^T [2 blocks of (64 dims x 32 keys)]
// (keys contiguous, the K-major B operand of O += P V), rounded to TF32, and
// with MODE 0 the residuals into a second V^T tile. Each warp moves 32
// consecutive keys of one 4-dim chunk per step, so the 32 scalar stores of a
// step (one dim, 32 keys) fall in 32 different banks.
template <int MODE, int NW>
__device__ __forceinline__ void transpose_v(const uint8_t* stage_v, uint8_t* vt, uint8_t* vt_lo, int t) {
  const int lane = t & 31, w = t >> 5;
#pragma unroll
  for (int u = 0; u < 32 / NW; ++u) {
    const int unit = w * (32 / NW) + u;  // 32 units: (key half, box, chunk)
    const int kh = unit >> 4, box = (unit >> 3) & 1, c = unit & 7;
    const int key = kh * 32 + lane;
    const float4 val = *reinterpret_cast<const float4*>(stage_v + box * (64 * 128) + key * 128 + ((c ^ (key & 7)) << 4));
    const float v4[4] = {val.x, val.y, val.z, val.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int d = box * 32 + c * 4 + e;
      const int off = kh * (64 * 128) + sw128(d, lane);
      const float hi = tf32_round(v4[e]);
      *reinterpret_cast<float*>(vt + off) = hi;
      if (MODE == 0) *reinterpret_cast<float*>(vt_lo + off) = v4[e] - hi;
    }
  }
}

// bf16 hi = round(v), lo = round(v - hi) of four consecutive values, as two
// 8-byte words of packed pairs.
__device__ __forceinline__ void split_bf16x4(float4 v, uint2& hi, uint2& lo) {
  const __nv_bfloat162 h0 = __floats2bfloat162_rn(v.x, v.y), h1 = __floats2bfloat162_rn(v.z, v.w);
  const float2 f0 = __bfloat1622float2(h0), f1 = __bfloat1622float2(h1);
  const float2 r0 = ub::fma2(make_float2(f0.x, f0.y), make_float2(-1.f, -1.f), make_float2(v.x, v.y));
  const float2 r1 = ub::fma2(make_float2(f1.x, f1.y), make_float2(-1.f, -1.f), make_float2(v.z, v.w));
  const __nv_bfloat162 l0 = __floats2bfloat162_rn(r0.x, r0.y);
  const __nv_bfloat162 l1 = __floats2bfloat162_rn(r1.x, r1.y);
  hi = make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
  lo = make_uint2(*reinterpret_cast<const uint32_t*>(&l0), *reinterpret_cast<const uint32_t*>(&l1));
}

// Byte offset of element (row r, column c < 64) of a [rows x 64] bf16 tile with
// 128-byte rows and the 128-byte swizzle (16-byte chunk index XOR row % 8).
__device__ __forceinline__ int sw128h(int r, int c) { return r * 128 + ((((c >> 3) ^ (r & 7))) << 4) + (c & 7) * 2; }

// MODE 2 operand preparation: the fp32 staging tile (2 boxes of [box_rows x 32
// dims], 128-byte swizzled rows) to bf16 hi / lo tiles [box_rows x 64 dims], with
// the optional rotary rotation of each (even, odd) dim pair at position pos0 + row,
// then the factor `mul`.
__device__ __forceinline__ void split_tile_bf16(const uint8_t* p, uint8_t* hi, uint8_t* lo, int t, int nt,
                                                int box_rows, int pos0, const float2* __restrict__ rope,
                                                int rope_len, int hd, float mul) {
  const float4* h = reinterpret_cast<const float4*>(p);
  const int n4 = box_rows * 16;
  for (int i = t; i < n4; i += nt) {
    float4 v = h[i];
    const int box = i / (box_rows * 8), within = i - box * (box_rows * 8);
    const int row = within >> 3;
    const int d0 = box * 32 + (((within & 7) ^ (row & 7)) << 2);
    if (rope && d0 < hd) {
      int pos = pos0 + row;
      pos = pos < rope_len ? pos : rope_len - 1;
      const float2 cs0 = __ldg(rope + (long long)pos * (hd >> 1) + (d0 >> 1));
      const float2 cs1 = __ldg(rope + (long long)pos * (hd >> 1) + (d0 >> 1) + 1);
      v = make_float4(v.x * cs0.x - v.y * cs0.y, v.x * cs0.y + v.y * cs0.x, v.z * cs1.x - v.w * cs1.y,
                      v.z * cs1.y + v.w * cs1.x);
    }
    v = make_float4(v.x * mul, v.y * mul, v.z * mul, v.w * mul);
    uint2 vh, vl;
    split_bf16x4(v, vh, vl);
    const int off = sw128h(row, d0);
    *reinterpret_cast<uint2*>(hi + off) = vh;
    *reinterpret_cast<uint2*>(lo + off) = vl;
  }
}

// MODE 2: V staging [2 boxes of (64 keys x 32 dims)] -> V^T hi / lo bf16 tiles [64
// dims x 64 keys] (keys contiguous). Lane l takes keys 2l and 2l + 1 of one 4-dim chunk
// per step, so each dim's hi and lo parts of the key pair leave as one packed 32-bit
// store (the 32 lanes of a store fill one 128-byte dim row).
template <int NW>
__device__ __forceinline__ void transpose_v_bf16(const uint8_t* stage_v, uint8_t* vt, uint8_t* vt_lo, int t) {
  const int lane = t & 31, w = t >> 5;
  const int k0 = 2 * lane;
#pragma unroll
  for (int u = 0; u < 16 / NW; ++u) {
    const int unit = w * (16 / NW) + u;  // 16 units: (box, chunk)
    const int box = unit >> 3, c = unit & 7;
    const uint8_t* src = stage_v + box * (64 * 128);
    const float4 va = *reinterpret_cast<const float4*>(src + k0 * 128 + ((c ^ (k0 & 7)) << 4));
    const float4 vb = *reinterpret_cast<const float4*>(src + (k0 + 1) * 128 + ((c ^ ((k0 + 1) & 7)) << 4));
    const float a4[4] = {va.x, va.y, va.z, va.w}, b4[4] = {vb.x, vb.y, vb.z, vb.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int d = box * 32 + c * 4 + e;
      const int off = sw128h(d, k0);
      const __nv_bfloat162 h2 = __floats2bfloat162_rn(a4[e], b4[e]);
      const float2 f = __bfloat1622float2(h2);
      const float2 r = ub::fma2(f, make_float2(-1.f, -1.f), make_float2(a4[e], b4[e]));
      const __nv_bfloat162 l2 = __floats2bfloat162_rn(r.x, r.y);
      *reinterpret_cast<uint32_t*>(vt + off) = *reinterpret_cast<const uint32_t*>(&h2);
      *reinterpret_cast<uint32_t*>(vt_lo + off) = *reinterpret_cast<const uint32_t*>(&l2);
    }
  }
}

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Softmax role for one 128-query tile, thread = query row `qrow` (TMEM lane quarter of
// its warp at lane_base). The running output O_acc (64 dims of this row) stays in
// registers: each key tile's P V product is folded in with CUDA-core FMAs
// (O_acc = O_acc * corr + O_tile), which keeps fp32 accuracy over thousands of keys.
// S / P of key tile j sit at TMEM column s_col + 64 (j & 1) (MODE 0: P lo at plo_col + 64
// (j & 1)), the tile's P V product at o_col; s_full and p_ready are 2-entry rings.
template <int MODE>
__device__ __forceinline__ void softmax_rows(const AttnArgs& a, uint32_t lane_base, uint32_t s_col, uint32_t plo_col,
                                             uint32_t o_col, uint64_t* s_full, uint64_t* p_ready, uint64_t* o_done,
                                             int nkv, int qrow, int h, int bi, int bo, int lane) {
  float m = -INFINITY, l = 0.f, corr_prev = 0.f;
  float oacc[64];
#pragma unroll
  for (int d = 0; d < 64; ++d) oacc[d] = 0.f;
  bool ok = true;
  auto fold_tile = [&](float corr) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t t0[32];
      tmem_ld32(lane_base + o_col + 32 * half, t0);
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const float2 o2 = ub::fma2(make_float2(oacc[32 * half + i], oacc[32 * half + i + 1]), make_float2(corr, corr),
                                   make_float2(__uint_as_float(t0[i]), __uint_as_float(t0[i + 1])));
        oacc[32 * half + i] = o2.x;
        oacc[32 * half + i + 1] = o2.y;
      }
    }
  };
  for (int j = 0; j < nkv && ok; ++j) {
    if (!__all_sync(0xffffffffu, mbar_wait(&s_full[j & 1], (j >> 1) & 1))) {
      ok = false;
      break;
    }
    tc_fence_after();
    uint32_t s0[32], s1[32];
    __syncwarp();
    tmem_ld32(lane_base + s_col + (j & 1) * BK, s0);
    tmem_ld32(lane_base + s_col + (j & 1) * BK + 32, s1);
    // Scores are already in log2 units (Q carries scale * log2(e)); keys past lk
    // (only in the last tile) are masked to -inf.
    const int kbase = j * BK;
    float mx = -INFINITY;
    if (kbase + BK <= a.lk) {
#pragma unroll
      for (int i = 0; i < 32; ++i) mx = fmaxf(mx, fmaxf(__uint_as_float(s0[i]), __uint_as_float(s1[i])));
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float v0 = kbase + i < a.lk ? __uint_as_float(s0[i]) : -INFINITY;
        const float v1 = kbase + 32 + i < a.lk ? __uint_as_float(s1[i]) : -INFINITY;
        s0[i] = __float_as_uint(v0);
        s1[i] = __float_as_uint(v1);
        mx = fmaxf(mx, fmaxf(v0, v1));
      }
    }
    const float m_new = fmaxf(m, mx);
    const float corr = ex2f(m - m_new);
    float sum = 0.f;
    float2 sum2 = make_float2(0.f, 0.f);
    // P = exp2(s - m_new) rounded to TF32 (hi) plus, in MODE 0, the residual
    // (lo), written to TMEM one 32-key half at a time. MODE 2: bf16 hi / lo
    // pairs (keys 2i, 2i + 1 in column i), hi over the S tile's first 32
    // columns and lo over the next 32.
    if (MODE == 2) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const uint32_t (&sh)[32] = half == 0 ? s0 : s1;
        uint32_t hp[16], lp[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 d = ub::fma2(make_float2(__uint_as_float(sh[2 * i]), __uint_as_float(sh[2 * i + 1])),
                                    make_float2(1.f, 1.f), make_float2(-m_new, -m_new));
          const float p0 = ex2f(d.x), p1 = ex2f(d.y);
          sum2 = ub::fma2(make_float2(p0, p1), make_float2(1.f, 1.f), sum2);
          const __nv_bfloat162 h2 = __floats2bfloat162_rn(p0, p1);
          const float2 f = __bfloat1622float2(h2);
          const float2 r = ub::fma2(f, make_float2(-1.f, -1.f), make_float2(p0, p1));
          const __nv_bfloat162 l2 = __floats2bfloat162_rn(r.x, r.y);
          hp[i] = *reinterpret_cast<const uint32_t*>(&h2);
          lp[i] = *reinterpret_cast<const uint32_t*>(&l2);
        }
        // Keys 32 half .. 32 half + 31: hi columns 16 half .., lo columns 32 + 16 half ...
        tmem_st16(lane_base + s_col + (j & 1) * BK + 16 * half, hp);
        tmem_st16(lane_base + s_col + (j & 1) * BK + 32 + 16 * half, lp);
      }
    }
#pragma unroll
    for (int half = 0; half < 2 && MODE != 2; ++half) {
      uint32_t (&sh)[32] = half == 0 ? s0 : s1;
      uint32_t lo[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float p = ex2f(__uint_as_float(sh[i]) - m_new);
        sum += p;
        const float hi = tf32_round(p);
        sh[i] = __float_as_uint(hi);
        lo[i] = __float_as_uint(p - hi);
      }
      tmem_st32(lane_base + s_col + (j & 1) * BK + 32 * half, sh);
      if (MODE == 0) tmem_st32(lane_base + plo_col + (j & 1) * BK + 32 * half, lo);
    }
    if (j > 0) {
      // Fold the previous tile's P V product (complete once o_done fires)
      // before P V of this tile may overwrite it. P(j) itself went into the S
      // tile of P(j-2), whose product was waited for one tile ago.
      if (!__all_sync(0xffffffffu, mbar_wait(o_done, (j - 1) & 1))) {
        ok = false;
        break;
      }
      tc_fence_after();
      fold_tile(corr_prev);
    }
    l = l * corr + (sum + (sum2.x + sum2.y));
    m = m_new;
    corr_prev = corr;
    tmem_st_wait();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&p_ready[j & 1]);
  }
  if (ok && nkv > 0) ok = __all_sync(0xffffffffu, mbar_wait(o_done, (nkv - 1) & 1));
  tc_fence_after();
  if (ok) {
    __syncwarp();
    fold_tile(corr_prev);
    if (qrow < a.lq) {
      float inv = 1.f / l;
      if (a.gate)
        inv *= __ldg(a.gate + (long long)bo * a.g_so + (long long)bi * a.g_si + (long long)qrow * a.g_sr + h);
      const long long off =
          (long long)bo * a.o_so + (long long)bi * a.o_si + (long long)qrow * a.o_sr + (long long)h * a.hd;
#pragma unroll
      for (int d = 0; d < 64; d += 4) {
        if (d < a.hd) {
          const float4 v = make_float4(oacc[d] * inv, oacc[d + 1] * inv, oacc[d + 2] * inv, oacc[d + 3] * inv);
          if (a.o_bf16) {
            __nv_bfloat162 p0 = __floats2bfloat162_rn(v.x, v.y);
            __nv_bfloat162 p1 = __floats2bfloat162_rn(v.z, v.w);
            uint2 packed;
            packed.x = *reinterpret_cast<uint32_t*>(&p0);
            packed.y = *reinterpret_cast<uint32_t*>(&p1);
            *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(a.o) + off + d) = packed;
          } else {
            *reinterpret_cast<float4*>(reinterpret_cast<float*>(a.o) + off + d) = v;
          }
        }
      }
    }
  }
}

template <int MODE>
__global__ void __launch_bounds__(NT, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap mapQ, const __grid_constant__ CUtensorMap mapK,
                        const __grid_constant__ CUtensorMap mapV, const __grid_constant__ AttnArgs a) {
  using L = AL<MODE>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sQlo = smem + L::Q_BYTES;
  uint8_t* sKV = smem + L::Q_TOTAL;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + L::STAGES * L::STAGE);
  // K and V travel in separate barrier rings over the same stage slots, so the
  // next K tile can land (and its QK^T start) while the P V of an older tile
  // still holds that slot's V.
  uint64_t* q_full = bars;
  uint64_t* q_ready = bars + 1;
  uint64_t* k_full = bars + 2;
  uint64_t* k_conv = k_full + L::STAGES;
  uint64_t* k_free = k_conv + L::STAGES;
  uint64_t* v_full = k_free + L::STAGES;
  uint64_t* v_conv = v_full + L::STAGES;
  uint64_t* v_free = v_conv + L::STAGES;
  uint64_t* s_full = v_free + L::STAGES;  // [2]
  uint64_t* p_ready = s_full + 2;          // [2]
  uint64_t* o_done = p_ready + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x % a.q_tiles;
  const int h = (blockIdx.x / a.q_tiles) % a.heads;
  const int z = blockIdx.x / (a.q_tiles * a.heads);
  const int bi = z % a.inner, bo = z / a.inner;
  const int q0 = qt * BQ;
  const int nkv = (a.lk + BK - 1) / BK;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_ready, 4);
    for (int s = 0; s < L::STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_conv[s], 2);
      mbar_init(&k_free[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_conv[s], 2);
      mbar_init(&v_free[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_ready[i], 4);
    }
    mbar_init(o_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, L::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // Q, then the K ring
      mbar_expect_tx(q_full, L::Q_BYTES);
      tma_load_5d(sQ, &mapQ, q_full, 0, h, q0, bi, bo);
      tma_load_5d(sQ + BQ * 128, &mapQ, q_full, 32, h, q0, bi, bo);
      for (int j = 0; j < nkv; ++j) {
        const int s = j % L::STAGES, r = j / L::STAGES;
        if (r > 0 && !mbar_wait(&k_free[s], (r - 1) & 1)) break;
        uint8_t* st = sKV + s * L::STAGE;
        mbar_expect_tx(&k_full[s], L::KV_BYTES);
        tma_load_5d(st + L::K_OFF, &mapK, &k_full[s], 0, h, j * BK, bi, bo);
        tma_load_5d(st + L::K_OFF + BK * 128, &mapK, &k_full[s], 32, h, j * BK, bi, bo);
      }
    } else if (lane == 1) {  // the V ring
      for (int j = 0; j < nkv; ++j) {
        const int s = j % L::STAGES, r = j / L::STAGES;
        if (r > 0 && !mbar_wait(&v_free[s], (r - 1) & 1)) break;
        uint8_t* st = sKV + s * L::STAGE;
        mbar_expect_tx(&v_full[s], L::KV_BYTES);
        tma_load_5d(st + L::V_OFF, &mapV, &v_full[s], 0, h, j * BK, bi, bo);
        tma_load_5d(st + L::V_OFF + BK * 128, &mapV, &v_full[s], 32, h, j * BK, bi, bo);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_s = instr_desc(2u, (uint32_t)BK);  // N = 64 keys
      constexpr uint32_t id_o = instr_desc(2u, 64u);           // N = 64 dims
      bool ok = mbar_wait(q_ready, 0);
      const uint32_t q_hi = smem_u32(sQ), q_lo = smem_u32(sQlo);
      auto issue_s = [&](int j) {
        const uint8_t* st = sKV + (j % L::STAGES) * L::STAGE;
        const uint32_t k_hi = smem_u32(st + L::K_OFF), k_lo = smem_u32(st + L::KLO_OFF);
        const uint32_t d = tmem + L::S_COL + (j & 1) * BK;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t qa = (i >> 2) * (BQ * 128) + (i & 3) * 32;
          const uint32_t ka = (i >> 2) * (BK * 128) + (i & 3) * 32;
          umma_tf32(d, smem_desc(q_hi + qa, 128), smem_desc(k_hi + ka, 128), id_s, i > 0 ? 1u : 0u);
          if (MODE == 0) {
            umma_tf32(d, smem_desc(q_hi + qa, 128), smem_desc(k_lo + ka, 128), id_s, 1u);
            umma_tf32(d, smem_desc(q_lo + qa, 128), smem_desc(k_hi + ka, 128), id_s, 1u);
          }
        }
        umma_commit(&s_full[j & 1]);
        umma_commit(&k_free[j % L::STAGES]);
      };
      if (ok) ok = mbar_wait(&k_conv[0], 0);
      if (ok) {
        tc_fence_after();
        issue_s(0);
      }
      for (int j = 0; j < nkv && ok; ++j) {
        if (j + 1 < nkv) {
          if (!mbar_wait(&k_conv[(j + 1) % L::STAGES], ((j + 1) / L::STAGES) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s(j + 1);
        }
        if (!mbar_wait(&p_ready[j & 1], (j >> 1) & 1) || !mbar_wait(&v_conv[j % L::STAGES], (j / L::STAGES) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int s = j % L::STAGES;
        const uint8_t* st = sKV + s * L::STAGE;
        const uint32_t vt_hi = smem_u32(st + L::VT_OFF), vt_lo = smem_u32(st + L::VTLO_OFF);
        const uint32_t p_hi = tmem + L::S_COL + (j & 1) * BK;
        const uint32_t p_lo = tmem + L::PLO_COL + (j & 1) * BK;
        const uint32_t o = tmem + L::O_COL;
#pragma unroll
        for (int i = 0; i < 8; ++i) {  // 8 keys per step
          const uint32_t vb = (i >> 2) * (64 * 128) + (i & 3) * 32;
          umma_tf32_ts(o, p_hi + 8 * i, smem_desc(vt_hi + vb, 128), id_o, i > 0 ? 1u : 0u);
          if (MODE == 0) {
            umma_tf32_ts(o, p_hi + 8 * i, smem_desc(vt_lo + vb, 128), id_o, 1u);
            umma_tf32_ts(o, p_lo + 8 * i, smem_desc(vt_hi + vb, 128), id_o, 1u);
          }
        }
        umma_commit(o_done);
        umma_commit(&v_free[s]);
      }
      if (!ok) atomicExch(&g_error_flag, 3);
    }
  } else if (warp >= 6) {
    // Operand preparation for Q (once) and every K/V tile.
    const int ct = threadIdx.x - 192;
    bool ok = mbar_wait(q_full, 0);
    if (ok) {
      split_tile<MODE>(sQ, sQlo, L::Q_BYTES / 16, ct, 128, BQ, q0, a.rope, a.rope_len, a.hd, a.c);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_ready);
    }
    // Warps 6-7 prepare K tiles, warps 8-9 V tiles.
    const bool k_role = warp < 8;
    const int rt = ct & 63;
    for (int j = 0; j < nkv && ok; ++j) {
      const int s = j % L::STAGES, r = j / L::STAGES;
      uint8_t* st = sKV + s * L::STAGE;
      if (k_role) {
        if (!mbar_wait(&k_full[s], r & 1)) break;
        split_tile<MODE>(st + L::K_OFF, st + L::KLO_OFF, L::KV_BYTES / 16, rt, 64, BK, j * BK, a.rope,
                         a.rope_len, a.hd, 1.0f);
      } else {
        if (!mbar_wait(&v_full[s], r & 1)) break;
        transpose_v<MODE, 2>(st + L::V_OFF, st + L::VT_OFF, st + (MODE == 0 ? L::VTLO_OFF : L::VT_OFF), rt);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(k_role ? &k_conv[s] : &v_conv[s]);
    }
  } else {
    // Softmax warps 2-5: thread = query row 32*(warp%4) + lane.
    const int qw = warp & 3;
    softmax_rows<MODE>(a, tmem + ((uint32_t)(qw * 32) << 16), L::S_COL, L::PLO_COL, L::O_COL, s_full, p_ready,
                       o_done, nkv, q0 + qw * 32 + lane, h, bi, bo, lane);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

// MODE 2 with two query tiles per CTA (256 queries of one head). Both tiles use every
// K / V tile (loaded and split once), and their softmax warp groups run concurrently,
// so one tile's softmax overlaps the other's MMAs: with a single query tile the chain
// S -> softmax -> P V of each key tile leaves the tensor pipe idle most of the time.
//   warp 0      TMA producer: lane 0 Q of tile A then the K ring, lane 1 the V ring,
//               lane 2 Q of tile B once tile A's staging is consumed
//   warp 1      MMA issue: S_A, S_B of key tile j + 1, then P_A V, P_B V of tile j
//   warps 2-5   softmax of query tile A, warps 6-9 of query tile B
//   warps 10-11 operand preparation: Q splits, then K split and V^T transpose of every key tile
constexpr int NT2 = 384;
struct AL2 {
  static constexpr int QS_BYTES = 2 * BQ * 128;       // fp32 Q staging (2 boxes of 32 dims)
  static constexpr int QH = BQ * 128;                 // one bf16 Q tile (128 rows x 64 dims)
  static constexpr int Q_TOTAL = QS_BYTES + 4 * QH;   // staging, A hi, A lo, B hi, B lo
  static constexpr int KV = 2 * BK * 128, TH = BK * 128;
  static constexpr int K_OFF = 0, KH_OFF = KV, KLO_OFF = KV + TH, V_OFF = KV + 2 * TH;
  static constexpr int VT_OFF = 2 * KV + 2 * TH, VTLO_OFF = VT_OFF + TH, STAGE = VTLO_OFF + TH;
  static constexpr int STAGES = 2;
  static constexpr int NBARS = 26;
  static constexpr int SMEM = Q_TOTAL + STAGES * STAGE + 1024 + 256;
  static constexpr int S_COL = 0;    // query tile t: S / P at 128 t + 64 (j & 1)
  static constexpr int O_COL = 256;  // query tile t: P V product at 256 + 64 t
  static constexpr int TMEM_COLS = 512;
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static_assert(NBARS * 8 + 4 <= 256, "barrier area");
};

__global__ void __launch_bounds__(NT2, 1)
    attention_tc_pair_kernel(const __grid_constant__ CUtensorMap mapQ, const __grid_constant__ CUtensorMap mapK,
                             const __grid_constant__ CUtensorMap mapV, const __grid_constant__ AttnArgs a) {
  using L = AL2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQs = smem;
  uint8_t* sKV = smem + L::Q_TOTAL;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + L::STAGES * L::STAGE);
  uint64_t* q_full = bars;        // phase 0: tile A landed, phase 1: tile B
  uint64_t* q_ready = bars + 1;   // [2]: hi / lo of tile t written
  uint64_t* q_free = bars + 3;    // staging of tile A consumed
  uint64_t* k_full = bars + 4;    // [2]
  uint64_t* k_conv = bars + 6;    // [2]
  uint64_t* k_free = bars + 8;    // [2]
  uint64_t* v_full = bars + 10;   // [2]
  uint64_t* v_conv = bars + 12;   // [2]
  uint64_t* v_free = bars + 14;   // [2]
  uint64_t* s_full = bars + 16;   // [tile][2]
  uint64_t* p_ready = bars + 20;  // [tile][2]
  uint64_t* o_done = bars + 24;   // [tile]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::NBARS);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q_pairs = (a.q_tiles + 1) / 2;
  const int qp = blockIdx.x % q_pairs;
  const int h = (blockIdx.x / q_pairs) % a.heads;
  const int z = blockIdx.x / (q_pairs * a.heads);
  const int bi = z % a.inner, bo = z / a.inner;
  const int q0 = qp * 2 * BQ;
  const int nq = q0 + BQ < a.lq ? 2 : 1;  // query tiles of this CTA (uniform)
  const int nkv = (a.lk + BK - 1) / BK;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(&q_ready[0], 2);
    mbar_init(&q_ready[1], 2);
    mbar_init(q_free, 2);
    for (int s = 0; s < L::STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_conv[s], 2);
      mbar_init(&k_free[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_conv[s], 2);
      mbar_init(&v_free[s], 1);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_ready[i], 4);
    }
    mbar_init(&o_done[0], 1);
    mbar_init(&o_done[1], 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, L::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // Q of tile A, then the K ring
      mbar_expect_tx(q_full, L::QS_BYTES);
      tma_load_5d(sQs, &mapQ, q_full, 0, h, q0, bi, bo);
      tma_load_5d(sQs + BQ * 128, &mapQ, q_full, 32, h, q0, bi, bo);
      for (int j = 0; j < nkv; ++j) {
        const int s = j % L::STAGES, r = j / L::STAGES;
        if (r > 0 && !mbar_wait(&k_free[s], (r - 1) & 1)) break;
        uint8_t* st = sKV + s * L::STAGE;
        mbar_expect_tx(&k_full[s], L::KV);
        tma_load_5d(st + L::K_OFF, &mapK, &k_full[s], 0, h, j * BK, bi, bo);
        tma_load_5d(st + L::K_OFF + BK * 128, &mapK, &k_full[s], 32, h, j * BK, bi, bo);
      }
    } else if (lane == 1) {  // the V ring
      for (int j = 0; j < nkv; ++j) {
        const int s = j % L::STAGES, r = j / L::STAGES;
        if (r > 0 && !mbar_wait(&v_free[s], (r - 1) & 1)) break;
        uint8_t* st = sKV + s * L::STAGE;
        mbar_expect_tx(&v_full[s], L::KV);
        tma_load_5d(st + L::V_OFF, &mapV, &v_full[s], 0, h, j * BK, bi, bo);
        tma_load_5d(st + L::V_OFF + BK * 128, &mapV, &v_full[s], 32, h, j * BK, bi, bo);
      }
    } else if (lane == 2 && nq == 2) {  // Q of tile B into the staging tile A has left
      if (mbar_wait(q_free, 0)) {
        mbar_expect_tx(q_full, L::QS_BYTES);
        tma_load_5d(sQs, &mapQ, q_full, 0, h, q0 + BQ, bi, bo);
        tma_load_5d(sQs + BQ * 128, &mapQ, q_full, 32, h, q0 + BQ, bi, bo);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_s = instr_desc(1u, (uint32_t)BK);  // kind::f16, N = 64 keys
      constexpr uint32_t id_o = instr_desc(1u, 64u);           // N = 64 dims
      bool ok = mbar_wait(&q_ready[0], 0) && (nq == 1 || mbar_wait(&q_ready[1], 0));
      auto issue_s = [&](int j) {
        const uint8_t* st = sKV + (j % L::STAGES) * L::STAGE;
        const uint32_t k_hi = smem_u32(st + L::KH_OFF), k_lo = smem_u32(st + L::KLO_OFF);
        for (int t = 0; t < nq; ++t) {
          const uint32_t q_hi = smem_u32(smem + L::QS_BYTES + 2 * t * L::QH), q_lo = q_hi + L::QH;
          const uint32_t d = tmem + L::S_COL + 128 * t + (j & 1) * BK;
#pragma unroll
          for (int i = 0; i < 4; ++i) {  // 16 dims per kind::f16 step
            umma_bf16(d, smem_desc(q_hi + 32 * i, 128), smem_desc(k_hi + 32 * i, 128), id_s, i > 0 ? 1u : 0u);
            umma_bf16(d, smem_desc(q_hi + 32 * i, 128), smem_desc(k_lo + 32 * i, 128), id_s, 1u);
            umma_bf16(d, smem_desc(q_lo + 32 * i, 128), smem_desc(k_hi + 32 * i, 128), id_s, 1u);
          }
          umma_commit(&s_full[2 * t + (j & 1)]);
        }
        umma_commit(&k_free[j % L::STAGES]);
      };
      if (ok) ok = mbar_wait(&k_conv[0], 0);
      if (ok) {
        tc_fence_after();
        issue_s(0);
      }
      for (int j = 0; j < nkv && ok; ++j) {
        if (j + 1 < nkv) {
          if (!mbar_wait(&k_conv[(j + 1) % L::STAGES], ((j + 1) / L::STAGES) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s(j + 1);
        }
        const int s = j % L::STAGES;
        if (!mbar_wait(&v_conv[s], (j / L::STAGES) & 1)) {
          ok = false;
          break;
        }
        const uint8_t* st = sKV + s * L::STAGE;
        const uint32_t vt_hi = smem_u32(st + L::VT_OFF), vt_lo = smem_u32(st + L::VTLO_OFF);
        for (int t = 0; t < nq && ok; ++t) {
          if (!mbar_wait(&p_ready[2 * t + (j & 1)], (j >> 1) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // P hi packed in the S tile's columns [0, 32), P lo in [32, 64): 16 keys per step.
          const uint32_t p_hi = tmem + L::S_COL + 128 * t + (j & 1) * BK;
          const uint32_t o = tmem + L::O_COL + 64 * t;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            umma_bf16_ts(o, p_hi + 8 * i, smem_desc(vt_hi + 32 * i, 128), id_o, i > 0 ? 1u : 0u);
            umma_bf16_ts(o, p_hi + 8 * i, smem_desc(vt_lo + 32 * i, 128), id_o, 1u);
            umma_bf16_ts(o, p_hi + 32 + 8 * i, smem_desc(vt_hi + 32 * i, 128), id_o, 1u);
          }
          umma_commit(&o_done[t]);
        }
        if (!ok) break;
        umma_commit(&v_free[s]);
      }
      if (!ok) atomicExch(&g_error_flag, 3);
    }
  } else if (warp >= 10) {
    // Operand preparation (64 threads): the Q tiles, then K and V^T of every key tile.
    const int ct = threadIdx.x - 320;
    bool ok = true;
    for (int t = 0; t < nq && ok; ++t) {
      ok = mbar_wait(q_full, t);
      if (!ok) break;
      uint8_t* qh = smem + L::QS_BYTES + 2 * t * L::QH;
      split_tile_bf16(sQs, qh, qh + L::QH, ct, 64, BQ, q0 + t * BQ, a.rope, a.rope_len, a.hd, a.c);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&q_ready[t]);
        if (t == 0) mbar_arrive(q_free);
      }
    }
    for (int j = 0; j < nkv && ok; ++j) {
      const int s = j % L::STAGES, r = j / L::STAGES;
      uint8_t* st = sKV + s * L::STAGE;
      if (!mbar_wait(&k_full[s], r & 1)) break;
      split_tile_bf16(st + L::K_OFF, st + L::KH_OFF, st + L::KLO_OFF, ct, 64, BK, j * BK, a.rope, a.rope_len, a.hd,
                      1.0f);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&k_conv[s]);
      if (!mbar_wait(&v_full[s], r & 1)) break;
      transpose_v_bf16<2>(st + L::V_OFF, st + L::VT_OFF, st + L::VTLO_OFF, ct);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&v_conv[s]);
    }
  } else {
    // Softmax warps 2-5 (tile A) and 6-9 (tile B): thread = query row 32*(warp%4) + lane.
    const int t = (warp - 2) >> 2, qw = warp & 3;
    if (t < nq)
      softmax_rows<2>(a, tmem + ((uint32_t)(qw * 32) << 16), L::S_COL + 128 * t, 0, L::O_COL + 64 * t,
                      &s_full[2 * t], &p_ready[2 * t], &o_done[t], nkv, q0 + t * BQ + qw * 32 + lane, h, bi, bo,
                      lane);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
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

// 5-D map (head dim, head, row, inner batch, outer batch) of one of Q/K/V
// with boxes of 32 dims x box_rows rows.
bool head_map(CUtensorMap* m, const float* base, int hd, int heads, int rows, int inner, int outer,
              long long row_stride, long long inner_stride, long long outer_stride, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[5] = {(cuuint64_t)hd, (cuuint64_t)heads, (cuuint64_t)rows, (cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[4] = {(cuuint64_t)hd * 4, (cuuint64_t)row_stride * 4, (cuuint64_t)inner_stride * 4,
                           (cuuint64_t)outer_stride * 4};
  cuuint32_t box[5] = {32, 1, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t es[5] = {1, 1, 1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 5, const_cast<float*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// A stride of a dimension of extent 1 is never used; give it a legal value.
long long legal_stride(long long s, int extent) { return extent == 1 && s <= 0 ? 4 : s; }

int attention_launch(const float* q, const float* k, const float* v, const UnblendAttnParams* p, int mode,
                     void* stream) {
  UB_REQUIRE(q && k && v && p && p->out && (mode == 0 || mode == 1 || mode == 2));
  UB_REQUIRE(p->outer > 0 && p->inner > 0 && p->heads > 0 && p->lq > 0 && p->lk > 0);
  UB_REQUIRE(p->hd > 0 && p->hd <= 64 && p->hd % 4 == 0);
  const long long q_so = legal_stride(p->q_so, p->outer), q_si = legal_stride(p->q_si, p->inner);
  const long long kv_so = legal_stride(p->kv_so, p->outer), kv_si = legal_stride(p->kv_si, p->inner);
  UB_REQUIRE(p->q_sr > 0 && p->kv_sr > 0 && q_so > 0 && q_si > 0 && kv_so > 0 && kv_si > 0);
  UB_REQUIRE(p->q_sr % 4 == 0 && q_so % 4 == 0 && q_si % 4 == 0 && p->kv_sr % 4 == 0 && kv_so % 4 == 0 &&
             kv_si % 4 == 0);
  UB_REQUIRE(p->o_sr % 4 == 0 && p->o_so % 4 == 0 && p->o_si % 4 == 0);
  UB_REQUIRE((reinterpret_cast<uintptr_t>(q) & 15) == 0 && (reinterpret_cast<uintptr_t>(k) & 15) == 0 &&
             (reinterpret_cast<uintptr_t>(v) & 15) == 0 && (reinterpret_cast<uintptr_t>(p->out) & 15) == 0);
  UB_REQUIRE(!p->rope || (p->rope_len > 0 && (reinterpret_cast<uintptr_t>(p->rope) & 7) == 0));
  CUtensorMap mq, mk, mv;
  if (!head_map(&mq, q, p->hd, p->heads, p->lq, p->inner, p->outer, p->q_sr, q_si, q_so, BQ) ||
      !head_map(&mk, k, p->hd, p->heads, p->lk, p->inner, p->outer, p->kv_sr, kv_si, kv_so, BK) ||
      !head_map(&mv, v, p->hd, p->heads, p->lk, p->inner, p->outer, p->kv_sr, kv_si, kv_so, BK))
    return UNBLEND_ERR_INVALID;
  AttnArgs a{};
  a.heads = p->heads;
  a.lq = p->lq;
  a.lk = p->lk;
  a.hd = p->hd;
  a.q_tiles = (p->lq + BQ - 1) / BQ;
  a.inner = p->inner;
  a.o = p->out;
  a.o_so = p->o_so;
  a.o_si = p->o_si;
  a.o_sr = p->o_sr;
  a.o_bf16 = p->out_bf16 ? 1 : 0;
  a.gate = p->gate;
  a.g_so = p->g_so;
  a.g_si = p->g_si;
  a.g_sr = p->g_sr;
  a.rope = reinterpret_cast<const float2*>(p->rope);
  a.rope_len = p->rope_len;
  a.c = p->scale * 1.4426950408889634f;
  const long long grid = (long long)p->outer * p->inner * p->heads * a.q_tiles;
  UB_REQUIRE(grid < (1LL << 31));
  cudaStream_t st = ub::as_stream(stream);
  if (mode == 0) {
    cudaFuncSetAttribute(attention_tc_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, AL<0>::SMEM);
    attention_tc_kernel<0><<<(unsigned)grid, NT, AL<0>::SMEM, st>>>(mq, mk, mv, a);
  } else if (mode == 2) {
    // Two query tiles per CTA (ceil(q_tiles / 2) CTAs per head and sequence).
    const long long grid2 = (long long)p->outer * p->inner * p->heads * ((a.q_tiles + 1) / 2);
    cudaFuncSetAttribute(attention_tc_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AL2::SMEM);
    attention_tc_pair_kernel<<<(unsigned)grid2, NT2, AL2::SMEM, st>>>(mq, mk, mv, a);
  } else {
    cudaFuncSetAttribute(attention_tc_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, AL<1>::SMEM);
    attention_tc_kernel<1><<<(unsigned)grid, NT, AL<1>::SMEM, st>>>(mq, mk, mv, a);
  }
  UB_CHECK_LAUNCH();
  return 0;
}

}  // namespace

extern "C" int unblend_attention_error_flag(int* out_host, int clear) {
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

extern "C" int unblend_attention_tc(const float* q, const float* k, const float* v, float* out, int batch, int heads,
                                    int lq, int lk, int hd, long long q_sb, long long q_sr, long long kv_sb,
                                    long long kv_sr, long long o_sb, long long o_sr, float scale, int mode,
                                    void* stream) {
  UnblendAttnParams p{};
  p.outer = batch;
  p.inner = 1;
  p.heads = heads;
  p.lq = lq;
  p.lk = lk;
  p.hd = hd;
  p.q_so = q_sb;
  p.q_si = 4;
  p.q_sr = q_sr;
  p.kv_so = kv_sb;
  p.kv_si = 4;
  p.kv_sr = kv_sr;
  p.out = out;
  p.o_so = o_sb;
  p.o_si = 0;
  p.o_sr = o_sr;
  p.scale = scale;
  return attention_launch(q, k, v, &p, mode, stream);
}

extern "C" int unblend_attention_tc2(const float* q, const float* k, const float* v, const UnblendAttnParams* p,
                                     int mode, void* stream) {
  return attention_launch(q, k, v, p, mode, stream);
}
