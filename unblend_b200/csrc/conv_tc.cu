// Implicit-GEMM convolution on the 5th-generation tensor cores (tcgen05).
//
// Same operation and parameter block as the SIMT path (UnblendConvParams):
// output positions (b, h, w) are the M dimension, output channels N, and the
// K dimension is walked tap by tap. Each K chunk of 32 input channels of one
// tap is a TMA box load of [m_box rows x 32 channels] from a 4-D tensor map of
// the channels-last input (C, W, H, B) at the tap's shifted coordinates; the
// hardware's out-of-bounds zero fill implements the convolution padding.
//
// Persistent: one CTA per SM walks the 128 x BN output tiles in a grid-stride
// loop, with the accumulator double-buffered in TMEM (2 x BN columns) so the
// epilogue of one tile overlaps the main loop of the next.
// Warp roles (448 threads):
//   warp 0    TMA producer (one elected lane)
//   warp 1    TMEM allocation + MMA issue (one elected lane)
//   warps 2-5 operand conversion in shared memory
//   warps 6-13 epilogue (two per TMEM lane quarter, alternate 32-column chunks)
// fp32 mode: each fp32 A tile is split in place into a TF32 "hi" part and a
// residual "lo" tile; weights come pre-split; D += Ahi*Bhi + Ahi*Blo + Alo*Bhi
// (3 x kind::tf32) keeps fp32-level accuracy. bf16 mode: the fp32 A tile is
// converted to bf16 and multiplied with bf16 weights (kind::f16). 3-pass bf16
// mode (MODE 2): the same three products with bf16 hi / lo parts (hi = x
// rounded to bf16, lo = x - hi rounded to bf16, 16 significant bits in all) in
// kind::f16, whose MMAs take 16 channels each instead of 8; MODE 4 is MODE 2 with
// the three taps of a 3-wide kernel row sharing one A load and split (tiles of up
// to 128 columns; a different K order, so not bit-identical). bf16-activation mode
// (MODE 3): the input is already bf16 in memory (written by the producing kernel
// for a consumer that multiplies in bf16), so TMA lands the A tile in its MMA
// layout and nothing is converted; otherwise as the bf16 mode.
// The accumulator lives in TMEM (128 lanes x BN fp32 columns); the epilogue
// reads it with tcgen05.ld and applies bias, GELU / GLU, the LayerScale
// residual and GroupNorm statistics, as the SIMT kernel does.
#include <cuda_bf16.h>
#include <cudaTypedefs.h>
#include <string.h>

#include "common.cuh"
#include "tc_common.cuh"

namespace {

using namespace ub::tc;

constexpr int MAXT = 16;
constexpr int NT = 448;
constexpr int EPI_WARPS = 8;

struct TcArgs {
  long long tiles;
  int B, H, W_out;
  int m_valid, m_box;
  int tiles_w, tiles_n;
  int n_out;
  int a_sh;
  int ntaps, nchunks;
  int tap_dh[MAXT], tap_dw[MAXT], tap_c0[MAXT], tap_clen[MAXT], tap_k0[MAXT];
  // Taps that read the same input rows shifted along w share one A load:
  // sub-tap 1 / 2 of load t use weight K offsets tap_k1/k2 and read the A tile
  // from row tap_s1/s2 on (sub-tap 0: row 0, offset tap_k0).
  int tap_n[MAXT], tap_k1[MAXT], tap_k2[MAXT], tap_s1[MAXT], tap_s2[MAXT];
  int a_rows;  // rows of each A load: m_box plus the largest sub-tap shift
  const float* bias;
  float* y;
  long long out_sb, out_sh, out_sw, out_sg;
  int n_group;
  int act;
  const float* res;
  const float* res_scale;
  double* stats;
  int stats_per_h;
  int tma_store;  // 1: whole 32-column chunks leave through TMA bulk tensor stores (no residual)
  const float* post;  // post-activation add: post[h * post_sh + output channel], or null
  long long post_sh;
  int y_bf16;  // 1: bf16 output through the bulk-store epilogue
};

// 3-pass TF32 tiles of up to 128 columns keep the A operand in TMEM: the
// converter warps write the TF32 hi / lo parts of each landed tile there
// (tcgen05.st) and the MMAs read A from TMEM, which issue faster than MMAs
// with both operands in shared memory when N <= 128.
template <int BN, int MODE>
struct ATmem {
  static constexpr bool value = MODE == 0 && BN <= 128;
};

// TMEM columns: the double-buffered accumulator (2 x BN), plus 64 columns
// (A hi, A lo) per pipeline stage with A in TMEM; rounded up to a power of two.
template <int BN, int MODE>
struct TmemCols {
  static constexpr int used = 2 * BN + (ATmem<BN, MODE>::value ? 4 * 64 : 0);
  static constexpr int value = used <= 128 ? 128 : used <= 256 ? 256 : 512;
  static_assert(used <= 512, "TMEM overflow");
};

// Channels per K chunk: 32 (128-byte fp32 rows, 128-byte swizzle), or 16 for the
// 3-pass TF32 mode with 256-column tiles, whose 96 KB stages would leave room for
// only two (64-byte rows, 64-byte swizzle, four stages). (192-column tiles keep
// 32-channel chunks and two stages: 16-channel chunks measured slower there.)
template <int BN, int MODE>
struct ChunkK {
  static constexpr int value = (MODE == 0 && BN == 256) ? 16 : 32;
};

// MODE 2 and MODE 4 are the 3-pass bf16 split; MODE 4 groups the taps of a
// 3-wide kernel row (below) on tiles of up to 128 columns.
__host__ __device__ constexpr bool bf16x3(int mode) { return mode == 2 || mode == 4; }

// Sub-taps per A load: the bf16 modes with tiles of up to 192 columns, and MODE 4
// (tiles of up to 128 columns: wider 3-pass tiles would leave room for one
// pipeline stage), group up to three taps along w (a 3-wide kernel row) onto one
// A load of 128 + 8 rows, each sub-tap's MMAs starting at its shifted row; the
// input tile then crosses from L2, and is converted, once per kernel row instead
// of once per tap.
template <int BN, int MODE>
struct SubTaps {
  static constexpr int value = (((MODE == 1 || MODE == 3) && BN <= 192) || (MODE == 4 && BN <= 128)) ? 3 : 1;
};

template <int BN, int MODE>
struct Layout {
  static constexpr int KC = ChunkK<BN, MODE>::value;
  static constexpr int NSUB = SubTaps<BN, MODE>::value;
  static constexpr int A_ROWS = NSUB > 1 ? 136 : 128;                 // 128 rows + shift headroom
  static constexpr int ROWB = KC * 4;                                 // fp32 bytes per staged row
  static constexpr int A_BYTES = MODE == 3 ? 0 : A_ROWS * ROWB;       // fp32 staging, A_ROWS x KC (none: MODE 3)
  // lo (fp32) or bf16 tile in shared memory (1 KB aligned); none with A in TMEM
  // (MODE 2: bf16 hi and lo tiles, AT_BYTES apart)
  static constexpr int AT_BYTES = (A_ROWS * 64 + 1023) / 1024 * 1024;
  static constexpr int AC_BYTES =
      ATmem<BN, MODE>::value ? 0 : MODE == 0 ? A_ROWS * ROWB : bf16x3(MODE) ? 2 * AT_BYTES : AT_BYTES;
  static constexpr int B_BYTES = MODE == 0 ? BN * ROWB : BN * 64;     // one weight tile
  static constexpr int B_TILES = (MODE == 1 || MODE == 3) ? 1 : 2;   // hi + lo, or bf16
  static constexpr int STAGE = A_BYTES + AC_BYTES + NSUB * B_TILES * B_BYTES;
  static constexpr int EPI_BYTES = EPI_WARPS * 32 * 32 * 4;  // one 32 x 32 fp32 transpose tile per epilogue warp
  static constexpr int STAGE_BUDGET = 232448 - EPI_BYTES - 1024 - 256;  // 227 KB per CTA
  static constexpr int STAGES = STAGE_BUDGET / STAGE > 4 ? 4 : STAGE_BUDGET / STAGE;
  static constexpr int A_COL = 2 * BN;  // first TMEM column of the A stages (A in TMEM)
  static_assert(!ATmem<BN, MODE>::value || STAGES == 4, "four A stages in TMEM");
  static_assert(STAGES >= 2, "at least two pipeline stages");
  static constexpr int SMEM = STAGES * STAGE + EPI_BYTES + 1024 /*align*/ + 256 /*barriers*/;
  static_assert(SMEM <= 232448, "shared memory per CTA");
};

__device__ __forceinline__ float gelu(float x) { return ub::gelu_erf(x); }

__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Activations of the bulk-store epilogue. MODE 1 (bf16 operands, results
// feeding bf16 GEMMs) uses the tanh form of GELU (Hendrycks & Gimpel 2016,
// within 5e-4 of the erf form) and sigmoid(x) = (1 + tanh(x/2)) / 2 on the
// hardware tanh; the fp32 modes keep the exact erf GELU and take the sigmoid
// from the hardware exp2 and reciprocal approximations (a few ulp; a correctly
// rounded reciprocal made the level-0 GLU rewrite epilogue-bound, 1.9 against
// 0.9 ms without the activation).
template <int MODE>
__device__ __forceinline__ float epi_gelu(float x) {
  if (MODE == 1 || MODE == 3) {
    const float z = 0.7978845608028654f * fmaf(0.044715f * x, x * x, x);
    return 0.5f * x * (1.0f + tanh_approx(z));
  }
  return ub::gelu_erf(x);
}

template <int MODE>
__device__ __forceinline__ float epi_sigmoid(float x) {
  if (MODE == 1 || MODE == 3) return fmaf(0.5f, tanh_approx(0.5f * x), 0.5f);
  return ub::sigmoid_approx(x);
}

struct TileCoord {
  int b, h, w0, n0;
};

// Tile t -> (batch, output row h, first output position w0, first channel n0);
// channel tiles fastest so that concurrently running CTAs share the input rows.
template <int BN>
__device__ __forceinline__ TileCoord tile_coord(const TcArgs& a, long long t) {
  TileCoord c;
  c.n0 = (int)(t % a.tiles_n) * BN;
  const long long m_tile = t / a.tiles_n;
  c.w0 = (int)(m_tile % a.tiles_w) * a.m_valid;
  const long long t2 = m_tile / a.tiles_w;
  c.h = (int)(t2 % a.H);
  c.b = (int)(t2 / a.H);
  return c;
}

template <int BN, int MODE>
__global__ void __launch_bounds__(NT, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
                   const __grid_constant__ CUtensorMap mapB2, const __grid_constant__ CUtensorMap mapO,
                   const __grid_constant__ TcArgs a) {
  using L = Layout<BN, MODE>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi_smem = smem + L::STAGES * L::STAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_smem + L::EPI_BYTES);
  uint64_t* conv = full + L::STAGES;
  uint64_t* empty = conv + L::STAGES;
  uint64_t* acc_full = empty + L::STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;      // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const long long tiles = a.tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < L::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 4);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], EPI_WARPS);
    }
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, TmemCols<BN, MODE>::value);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nk = a.nchunks;

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t bytes_a = (uint32_t)(a.a_rows * (MODE == 3 ? 64 : L::ROWB));
      int it = 0;
      bool ok = true;
      for (long long t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const TileCoord c = tile_coord<BN>(a, t);
        for (int tap = 0; tap < a.ntaps && ok; ++tap) {
          const int ca = a.tap_c0[tap], wa = c.w0 + a.tap_dw[tap], ha = c.h * a.a_sh + a.tap_dh[tap];
          const int kb = a.tap_k0[tap], ns = a.tap_n[tap];
          const uint32_t bytes = bytes_a + (uint32_t)(ns * L::B_TILES * L::B_BYTES);
          for (int cc = 0; cc < a.tap_clen[tap] && ok; cc += L::KC, ++it) {
            const int s = it % L::STAGES;
            const int r = it / L::STAGES;
            if (r > 0 && !mbar_wait(&empty[s], (r - 1) & 1)) {
              ok = false;
              break;
            }
            uint8_t* st = smem + s * L::STAGE;
            mbar_expect_tx(&full[s], bytes);
            tma_load_4d(st, &mapA, &full[s], ca + cc, wa, ha, c.b);
            uint8_t* sb = st + L::A_BYTES + L::AC_BYTES;
            // Sub-tap u's weight tile(s) at sb + u * B_TILES * B_BYTES (hi, then lo for the split modes).
            tma_load_2d(sb, &mapB, &full[s], kb + cc, c.n0);
            if (MODE == 0 || bf16x3(MODE)) tma_load_2d(sb + L::B_BYTES, &mapB2, &full[s], kb + cc, c.n0);
#pragma unroll
            for (int u = 1; u < L::NSUB; ++u) {
              if (u >= ns) break;
              const int ku = (u == 1 ? a.tap_k1[tap] : a.tap_k2[tap]) + cc;
              uint8_t* su = sb + u * L::B_TILES * L::B_BYTES;
              tma_load_2d(su, &mapB, &full[s], ku, c.n0);
              if (L::B_TILES == 2) tma_load_2d(su + L::B_BYTES, &mapB2, &full[s], ku, c.n0);
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc(MODE == 0 ? 2u : 1u, (uint32_t)BN);  // kind::tf32 or bf16
      bool ok = true;
      int it = 0, i = 0;
      for (long long t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++i) {
        const int buf = i & 1, u = i >> 1;
        if (u > 0 && !mbar_wait(&acc_empty[buf], (u - 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * BN);
        // K steps with real channels in the current chunk: a chunk holds KC channels
        // of one tap, and the last chunk of a tap may be partly past c_in (zero fill,
        // e.g. 16 of 32 for 48-channel layers); the MMAs of all-zero steps are skipped.
        int tap = 0, cc = 0;
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int valid = min(L::KC, a.tap_clen[tap] - cc);
          const int ctap = tap;
          cc += L::KC;
          if (cc >= a.tap_clen[tap]) {
            cc = 0;
            ++tap;
          }
          const int s = it % L::STAGES;
          const int r = it / L::STAGES;
          if (!mbar_wait(&conv[s], r & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint8_t* st = smem + s * L::STAGE;
          const uint32_t sa = smem_u32(st);
          const uint32_t sac = sa + L::A_BYTES;
          const uint32_t sb = sac + L::AC_BYTES;
          if (ATmem<BN, MODE>::value) {
            // A hi / lo of this stage sit in TMEM columns [A_COL + 64 s, + 64).
            const uint32_t at = tmem + (uint32_t)(L::A_COL + 64 * s);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              if (j > 0 && 8 * j >= valid) break;
              const uint64_t dbh = smem_desc(sb + 32 * j, 128), dbl = smem_desc(sb + L::B_BYTES + 32 * j, 128);
              umma_tf32_ts(d, at + 8 * j, dbh, idesc, (kc > 0 || j > 0) ? 1u : 0u);
              umma_tf32_ts(d, at + 8 * j, dbl, idesc, 1u);
              umma_tf32_ts(d, at + 32 + 8 * j, dbh, idesc, 1u);
            }
          } else if (MODE == 0) {
#pragma unroll
            for (int j = 0; j < L::KC / 8; ++j) {
              if (j > 0 && 8 * j >= valid) break;  // 8 channels per kind::tf32 step
              const uint64_t dah = smem_desc(sa + 32 * j, L::ROWB), dal = smem_desc(sac + 32 * j, L::ROWB);
              const uint64_t dbh = smem_desc(sb + 32 * j, L::ROWB);
              const uint64_t dbl = smem_desc(sb + L::B_BYTES + 32 * j, L::ROWB);
              umma_tf32(d, dah, dbh, idesc, (kc > 0 || j > 0) ? 1u : 0u);
              umma_tf32(d, dah, dbl, idesc, 1u);
              umma_tf32(d, dal, dbh, idesc, 1u);
            }
          } else if (bf16x3(MODE)) {
            // Sub-tap u reads the hi / lo tiles from row shift_u on (64-byte rows).
            const int ns = L::NSUB > 1 ? a.tap_n[ctap] : 1;
#pragma unroll
            for (int u = 0; u < L::NSUB; ++u) {
              if (u >= ns) break;
              const int shift = u == 0 ? 0 : u == 1 ? a.tap_s1[ctap] : a.tap_s2[ctap];
              const uint32_t au = sac + (uint32_t)(64 * shift), bu = sb + (uint32_t)(u * 2 * L::B_BYTES);
#pragma unroll
              for (int j = 0; j < 2; ++j) {
                if (j > 0 && 16 * j >= valid) break;  // 16 channels per kind::f16 step
                const uint64_t dah = smem_desc(au + 32 * j, 64), dal = smem_desc(au + L::AT_BYTES + 32 * j, 64);
                const uint64_t dbh = smem_desc(bu + 32 * j, 64), dbl = smem_desc(bu + L::B_BYTES + 32 * j, 64);
                umma_bf16(d, dah, dbh, idesc, (kc > 0 || j > 0 || u > 0) ? 1u : 0u);
                umma_bf16(d, dah, dbl, idesc, 1u);
                umma_bf16(d, dal, dbh, idesc, 1u);
              }
            }
          } else {
            // Sub-tap u reads the bf16 A tile from row shift_u on (64-byte rows).
            const int ns = L::NSUB > 1 ? a.tap_n[ctap] : 1;
#pragma unroll
            for (int u = 0; u < L::NSUB; ++u) {
              if (u >= ns) break;
              const int shift = u == 0 ? 0 : u == 1 ? a.tap_s1[ctap] : a.tap_s2[ctap];
              const uint32_t au = sac + (uint32_t)(64 * shift), bu = sb + (uint32_t)(u * L::B_BYTES);
#pragma unroll
              for (int j = 0; j < 2; ++j) {
                if (j > 0 && 16 * j >= valid) break;  // 16 channels per kind::f16 step
                const uint64_t da = smem_desc(au + 32 * j, 64), db = smem_desc(bu + 32 * j, 64);
                umma_bf16(d, da, db, idesc, (kc > 0 || j > 0 || u > 0) ? 1u : 0u);
              }
            }
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&acc_full[buf]);
      }
      if (!ok) atomicExch(&g_error_flag, 2);
    }
  } else if (warp < 6) {
    // Converter warps 2-5: split / pack each landed A tile for the MMA.
    const int ct = threadIdx.x - 64;  // 0..127
    int it = 0;
    bool ok = true;
    for (long long t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
      for (int kc = 0; kc < nk; ++kc, ++it) {
        const int s = it % L::STAGES;
        const int r = it / L::STAGES;
        if (!mbar_wait(&full[s], r & 1)) {
          ok = false;
          break;
        }
        uint8_t* st = smem + s * L::STAGE;
        if (ATmem<BN, MODE>::value) {
          // Thread = tile row (its warp's TMEM lane quarter): the row's 32 fp32
          // values from the 128-byte swizzled tile, split, stored as 32 hi and
          // 32 lo columns. The TMA wrote this stage only after the MMAs that read
          // the stage's previous A columns completed (empty barrier), so the
          // columns are free.
          const int quarter = warp & 3;
          const int row = quarter * 32 + lane;
          const uint8_t* src = st + row * 128;
          uint32_t hv[32], lv[32];
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const float4 v = *reinterpret_cast<const float4*>(src + ((c ^ (row & 7)) << 4));
            const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float h = __uint_as_float((__float_as_uint(e[k]) + 0x1000u) & 0xFFFFE000u);
              hv[4 * c + k] = __float_as_uint(h);
              lv[4 * c + k] = __float_as_uint(e[k] - h);
            }
          }
          const uint32_t ta = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(L::A_COL + 64 * s);
          tmem_st32(ta, hv);
          tmem_st32(ta + 32, lv);
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&conv[s]);
          continue;
        }
        if (MODE == 0) {
          float4* hi = reinterpret_cast<float4*>(st);
          float4* lo = reinterpret_cast<float4*>(st + L::A_BYTES);
#pragma unroll
          for (int k = ct; k < 128 * L::KC / 4; k += 128) {
            const float4 v = hi[k];
            // hi = v rounded to the nearest TF32 value (ties away from zero), lo = v - hi exactly.
            float4 vh;
            vh.x = __uint_as_float((__float_as_uint(v.x) + 0x1000u) & 0xFFFFE000u);
            vh.y = __uint_as_float((__float_as_uint(v.y) + 0x1000u) & 0xFFFFE000u);
            vh.z = __uint_as_float((__float_as_uint(v.z) + 0x1000u) & 0xFFFFE000u);
            vh.w = __uint_as_float((__float_as_uint(v.w) + 0x1000u) & 0xFFFFE000u);
            hi[k] = vh;
            lo[k] = make_float4(v.x - vh.x, v.y - vh.y, v.z - vh.z, v.w - vh.w);
          }
        } else if (MODE == 3) {
          // The TMA wrote the bf16 tile in its MMA layout: nothing to convert.
        } else if (bf16x3(MODE)) {
          // hi = bf16(v), lo = bf16(v - hi): both written as 64-byte swizzled bf16 tiles.
          const uint8_t* src = st;
          uint8_t* dst = st + L::A_BYTES;
#pragma unroll
          for (int k = ct; k < L::A_ROWS * 8; k += 128) {
            const int row = k >> 3, c = k & 7;
            const float4 v = *reinterpret_cast<const float4*>(src + row * 128 + ((c ^ (row & 7)) << 4));
            const __nv_bfloat162 h0 = __floats2bfloat162_rn(v.x, v.y);
            const __nv_bfloat162 h1 = __floats2bfloat162_rn(v.z, v.w);
            const float2 f0 = __bfloat1622float2(h0), f1 = __bfloat1622float2(h1);
            const __nv_bfloat162 l0 = __floats2bfloat162_rn(v.x - f0.x, v.y - f0.y);
            const __nv_bfloat162 l1 = __floats2bfloat162_rn(v.z - f1.x, v.w - f1.y);
            const int off = row * 64 + (((c >> 1) ^ ((row >> 1) & 3)) << 4) + (c & 1) * 8;
            *reinterpret_cast<uint2*>(dst + off) =
                make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
            *reinterpret_cast<uint2*>(dst + L::AT_BYTES + off) =
                make_uint2(*reinterpret_cast<const uint32_t*>(&l0), *reinterpret_cast<const uint32_t*>(&l1));
          }
        } else {
          const uint8_t* src = st;
          uint8_t* dst = st + L::A_BYTES;
#pragma unroll
          for (int k = ct; k < L::A_ROWS * 8; k += 128) {
            const int row = k >> 3, c = k & 7;
            const float4 v = *reinterpret_cast<const float4*>(src + row * 128 + ((c ^ (row & 7)) << 4));
            __nv_bfloat162 p0 = __floats2bfloat162_rn(v.x, v.y);
            __nv_bfloat162 p1 = __floats2bfloat162_rn(v.z, v.w);
            uint2 packed;
            packed.x = *reinterpret_cast<uint32_t*>(&p0);
            packed.y = *reinterpret_cast<uint32_t*>(&p1);
            *reinterpret_cast<uint2*>(dst + row * 64 + (((c >> 1) ^ ((row >> 1) & 3)) << 4) + (c & 1) * 8) = packed;
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[s]);
      }
    }
  } else {
    // Epilogue warps 6-13: TMEM -> registers -> shared-memory transpose -> fused
    // ops -> global. After the transpose each lane owns 4 consecutive output
    // channels of 8 rows, so bias / scale loads are one float4 per lane and
    // each store instruction of the warp writes 4 whole row segments.
    const int q = warp & 3;  // TMEM lane quarter this warp may read
    float4* stage = reinterpret_cast<float4*>(epi_smem + (warp - 6) * 4096);
    const int c_first = 32 * ((warp - 6) >> 2);  // this warp's first chunk; the pair alternates chunks
    const int ch = lane & 7;
    const bool glu = a.act == UNBLEND_ACT_GLU;
    int i = 0;
    for (long long t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
      const TileCoord tc = tile_coord<BN>(a, t);
      const int b = tc.b, h = tc.h, w0 = tc.w0, n0 = tc.n0;
      const int buf = i & 1, u = i >> 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[buf], u & 1))) break;
      tc_fence_after();
      const uint32_t base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN);
      double s1 = 0.0, s2 = 0.0;  // per-lane statistics: fp32 partials of 4 values, summed in double
#pragma unroll 1
      for (int c0 = c_first; c0 < BN; c0 += 64) {
        if (n0 + c0 >= a.n_out) break;  // uniform across the warp
        uint32_t acc[32];
        __syncwarp();
        tmem_ld32(base + (uint32_t)c0, acc);
        if (a.tma_store && n0 + c0 + 32 <= a.n_out) {
          // Whole chunk, lane = output position: bias, activation, GLU and the
          // statistics in registers, one swizzled staging row per lane, then
          // bulk tensor stores of 16-row halves inside the tile's valid rows.
          const int row = q * 32 + lane;
          const bool rv = row < a.m_valid && w0 + row < a.W_out;
          float v[32];
          if (a.bias) {
            const float4* bp = reinterpret_cast<const float4*>(a.bias + n0 + c0);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 b4 = __ldg(bp + j);
              v[4 * j] = __uint_as_float(acc[4 * j]) + b4.x;
              v[4 * j + 1] = __uint_as_float(acc[4 * j + 1]) + b4.y;
              v[4 * j + 2] = __uint_as_float(acc[4 * j + 2]) + b4.z;
              v[4 * j + 3] = __uint_as_float(acc[4 * j + 3]) + b4.w;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(acc[j]);
          }
          if (a.act == UNBLEND_ACT_GELU) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = epi_gelu<MODE>(v[j]);
          }
          const int nv = glu ? 16 : 32;
          if (glu) {
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = v[2 * j] * epi_sigmoid<MODE>(v[2 * j + 1]);
          }
          if (a.post) {
            const float* pp = a.post + (long long)h * a.post_sh + (glu ? (n0 + c0) / 2 : n0 + c0);
            if ((reinterpret_cast<uintptr_t>(pp) & 15) == 0) {
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                if (4 * j < nv) {
                  const float4 p4 = __ldg(reinterpret_cast<const float4*>(pp) + j);
                  v[4 * j] += p4.x;
                  v[4 * j + 1] += p4.y;
                  v[4 * j + 2] += p4.z;
                  v[4 * j + 3] += p4.w;
                }
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (j < nv) v[j] += __ldg(pp + j);
            }
          }
          if (a.stats && rv) {
            float t1 = 0.f, t2 = 0.f;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (j < nv) {
                t1 += v[j];
                t2 += v[j] * v[j];
              }
            }
            s1 += t1;
            s2 += t2;
          }
          uint8_t* stg = reinterpret_cast<uint8_t*>(stage);
          if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
          __syncwarp();
          const int rb = a.y_bf16 ? 64 : nv * 4;     // staging row bytes: 128 or 64
          const int swz = ((lane * rb) >> 7) & ((rb >> 4) - 1);
          if (a.y_bf16) {
            // 32 values -> 16 bf16 pairs, four 16-byte units of a 64-byte row.
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              uint32_t u[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                __nv_bfloat162 pr = __floats2bfloat162_rn(v[8 * j + 2 * e], v[8 * j + 2 * e + 1]);
                u[e] = *reinterpret_cast<uint32_t*>(&pr);
              }
              *reinterpret_cast<uint4*>(stg + lane * rb + ((j ^ swz) << 4)) = make_uint4(u[0], u[1], u[2], u[3]);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              if (j < (nv >> 2))
                *reinterpret_cast<float4*>(stg + lane * rb + ((j ^ swz) << 4)) =
                    make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            const int xcol = glu ? (n0 + c0) / 2 : n0 + c0;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
              const int r0 = q * 32 + 16 * half;
              if (r0 < a.m_valid && w0 + r0 < a.W_out) {
                asm volatile(
                    "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                        &mapO),
                    "r"(smem_u32(stg + half * 16 * rb)), "r"(xcol), "r"(w0 + r0), "r"(h), "r"(b)
                    : "memory");
              }
            }
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          }
          continue;
        }
        if (a.tma_store) {
          if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
          __syncwarp();
        }
#pragma unroll
        for (int j = 0; j < 8; ++j)
          stage[lane * 8 + (j ^ (lane & 7))] =
              make_float4(__uint_as_float(acc[4 * j]), __uint_as_float(acc[4 * j + 1]),
                          __uint_as_float(acc[4 * j + 2]), __uint_as_float(acc[4 * j + 3]));
        __syncwarp();
        const int n = n0 + c0 + ch * 4;  // first of this lane's 4 accumulator columns
        const int nvalid = min(4, a.n_out - n);
        float4 bv = make_float4(0.f, 0.f, 0.f, 0.f);
        if (a.bias && nvalid > 0) {
          if (nvalid == 4) {
            bv = __ldg(reinterpret_cast<const float4*>(a.bias + n));
          } else {
            bv.x = __ldg(a.bias + n);
            if (nvalid > 1) bv.y = __ldg(a.bias + n + 1);
            if (nvalid > 2) bv.z = __ldg(a.bias + n + 2);
          }
        }
        const int nb = glu ? n / 2 : n;  // first output channel
        const int ocnt = glu ? nvalid / 2 : nvalid;
        const long long goff = (long long)(nb / a.n_group) * a.out_sg + (nb % a.n_group);
        const long long rowbase = (long long)b * a.out_sb + (long long)h * a.out_sh + goff;
        float4 sc = make_float4(1.f, 1.f, 1.f, 1.f);
        if (a.res && a.res_scale && ocnt > 0) {
          sc.x = __ldg(a.res_scale + nb);
          if (ocnt > 1) sc.y = __ldg(a.res_scale + nb + 1);
          if (ocnt > 2) sc.z = __ldg(a.res_scale + nb + 2);
          if (ocnt > 3) sc.w = __ldg(a.res_scale + nb + 3);
        }
        // Residual values of the lane's 8 rows, all loads in flight at once.
        float4 rv[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          rv[k] = make_float4(0.f, 0.f, 0.f, 0.f);
          const int row = q * 32 + k * 4 + (lane >> 3);
          const int wpos = w0 + row;
          if (a.res && ocnt > 0 && row < a.m_valid && wpos < a.W_out) {
            const float* rp = a.res + rowbase + (long long)wpos * a.out_sw;
            if (ocnt == 4) {
              rv[k] = *reinterpret_cast<const float4*>(rp);
            } else {
              rv[k].x = rp[0];
              if (ocnt > 1) rv[k].y = rp[1];
              if (ocnt > 2) rv[k].z = rp[2];
            }
          }
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int r = k * 4 + (lane >> 3);
          const int row = q * 32 + r;
          const int wpos = w0 + row;
          const float4 v = stage[r * 8 + (ch ^ (r & 7))];
          if (ocnt <= 0 || row >= a.m_valid || wpos >= a.W_out) continue;
          float x[4] = {v.x + bv.x, v.y + bv.y, v.z + bv.z, v.w + bv.w};
          if (a.act == UNBLEND_ACT_GELU) {
#pragma unroll
            for (int e = 0; e < 4; ++e) x[e] = gelu(x[e]);
          }
          float o[4];
          if (glu) {
            o[0] = x[0] * ub::sigmoid_approx(x[1]);
            o[1] = x[2] * ub::sigmoid_approx(x[3]);
            o[2] = o[3] = 0.f;
          } else {
            o[0] = x[0];
            o[1] = x[1];
            o[2] = x[2];
            o[3] = x[3];
          }
          if (a.post) {
            const float* pp = a.post + (long long)h * a.post_sh + nb;
#pragma unroll
            for (int e = 0; e < 4; ++e)
              if (e < ocnt) o[e] += __ldg(pp + e);
          }
          if (a.res) {
            o[0] = rv[k].x + sc.x * o[0];
            o[1] = rv[k].y + sc.y * o[1];
            o[2] = rv[k].z + sc.z * o[2];
            o[3] = rv[k].w + sc.w * o[3];
          }
          float* yp = a.y + rowbase + (long long)wpos * a.out_sw;
          if (ocnt == 4) {
            *reinterpret_cast<float4*>(yp) = make_float4(o[0], o[1], o[2], o[3]);
          } else if (ocnt == 2 && glu) {
            *reinterpret_cast<float2*>(yp) = make_float2(o[0], o[1]);
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e)
              if (e < ocnt) yp[e] = o[e];
          }
          float t1 = 0.f, t2 = 0.f;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            if (e < ocnt) {
              t1 += o[e];
              t2 += o[e] * o[e];
            }
          }
          s1 += t1;
          s2 += t2;
        }
      }
      // The accumulator buffer is free once every lane has read its columns.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      if (a.stats) {
        s1 = ub::warp_sum_d(s1);
        s2 = ub::warp_sum_d(s2);
        if (lane == 0) {
          const int g = a.stats_per_h ? b * a.H + h : b;
          atomicAdd(a.stats + 2 * g, s1);
          atomicAdd(a.stats + 2 * g + 1, s2);
        }
      }
    }
    if (a.tma_store && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TmemCols<BN, MODE>::value);
  }
}

// ---------------------------------------------------------------- host side

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

bool make_map(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* base, const cuuint64_t* dims,
              const cuuint64_t* strides_bytes, const cuuint32_t* box, CUtensorMapSwizzle sw) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(m, dt, (cuuint32_t)rank, const_cast<void*>(base), dims, strides_bytes, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int BN, int MODE>
int launch(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mb2, const CUtensorMap& mo,
           const TcArgs& args, long long tiles, cudaStream_t st) {
  using L = Layout<BN, MODE>;
  auto k = conv_tc_kernel<BN, MODE>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM);
  int dev = 0, sms = ub::kNumSMs;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const unsigned grid = (unsigned)(tiles < sms ? tiles : sms);
  k<<<grid, NT, L::SMEM, st>>>(ma, mb, mb2, mo, args);
  UB_CHECK_LAUNCH();
  return 0;
}

}  // namespace

extern "C" int unblend_error_flag(int* out_host, int clear) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, ub::tc::g_error_flag, sizeof(int));
  if (e != cudaSuccess) return (int)e;
  if (out_host) *out_host = v;
  if (clear) {
    int z = 0;
    e = cudaMemcpyToSymbol(ub::tc::g_error_flag, &z, sizeof(int));
    if (e != cudaSuccess) return (int)e;
  }
  return 0;
}

extern "C" int unblend_conv2d_tc(const void* x, const void* w_hi, const void* w_lo, const float* bias, float* y,
                                 const UnblendConvParams* p, int mode, int block_n, void* stream) {
  UB_REQUIRE(x && w_hi && y && p && mode >= 0 && mode <= 4);
  UB_REQUIRE(mode != 4 || block_n <= 128);  // shared tap loads: tiles of up to 128 columns
  UB_REQUIRE((mode == 3) == (p->x_bf16 != 0));  // mode 3 takes bf16 activations, the others fp32
  UB_REQUIRE(mode == 1 || mode == 3 || w_lo);  // the split modes take hi and lo weights
  UB_REQUIRE(block_n == 64 || block_n == 96 || block_n == 128 || block_n == 192 || block_n == 256);
  UB_REQUIRE(p->prologue == UNBLEND_PRO_NONE);
  UB_REQUIRE(p->c_in % 8 == 0 && p->c_in >= 16);
  UB_REQUIRE(p->n_group % 4 == 0 && p->out_sg % 4 == 0 && p->out_sw % 4 == 0 && p->out_sh % 4 == 0 &&
             p->out_sb % 4 == 0);
  UB_REQUIRE(p->act != UNBLEND_ACT_GLU || p->n_out % 2 == 0);
  UB_REQUIRE(p->in_sw == p->c_in && p->in_sh % 4 == 0 && p->in_sb % 4 == 0);
  // bf16 rows: 16-byte aligned row starts for the tensor map, unit stride only.
  UB_REQUIRE(mode != 3 || (p->sw == 1 && p->c_in % 8 == 0 && p->in_sh % 8 == 0 && p->in_sb % 8 == 0 &&
                           (reinterpret_cast<uintptr_t>(x) & 15) == 0));
  UB_REQUIRE(!bias || (reinterpret_cast<uintptr_t>(bias) & 15) == 0);
  UB_REQUIRE((reinterpret_cast<uintptr_t>(y) & 15) == 0 && (!p->res || (reinterpret_cast<uintptr_t>(p->res) & 15) == 0));
  UB_REQUIRE(p->act != UNBLEND_ACT_GLU || p->n_out % 4 == 0);
  TcArgs a{};
  a.B = p->batch;
  a.H = p->h_out;
  a.W_out = p->w_out;
  a.n_out = p->n_out;
  a.bias = bias;
  a.y = y;
  a.out_sb = p->out_sb;
  a.out_sh = p->out_sh;
  a.out_sw = p->out_sw;
  a.out_sg = p->out_sg;
  a.n_group = p->n_group;
  a.act = p->act;
  a.res = p->res;
  a.res_scale = p->res_scale;
  a.stats = p->stats;
  a.stats_per_h = p->stats_per_h;
  a.post = p->post;
  a.post_sh = p->post_sh;
  a.y_bf16 = p->y_bf16 ? 1 : 0;
  UB_REQUIRE(!a.y_bf16 || (p->act != UNBLEND_ACT_GLU && !p->res && p->n_out % 32 == 0 && p->n_group >= p->n_out &&
                           p->out_sw % 8 == 0 && p->out_sh % 8 == 0 && p->out_sb % 8 == 0));

  // A operand tensor map (C, W, H, B) and the tap table.
  CUtensorMap ma, mb, mb2;
  cuuint64_t dims[4];
  cuuint64_t strides[3];
  int kw_taps = p->kw, kh_taps = p->kh;
  int max_shift = 0;  // largest sub-tap row shift (rows of each A load past the tile's)
  const long long K = (long long)p->kh * p->kw * p->c_in;
  int nt = 0;
  if (p->sw == 1) {
    dims[0] = (cuuint64_t)p->c_in;
    dims[1] = (cuuint64_t)p->w_in;
    dims[2] = (cuuint64_t)p->h_in;
    dims[3] = (cuuint64_t)p->batch;
    const cuuint64_t es = mode == 3 ? 2 : 4;  // input element bytes
    strides[0] = (cuuint64_t)p->in_sw * es;
    strides[1] = (cuuint64_t)p->in_sh * es;
    strides[2] = (cuuint64_t)p->in_sb * es;
    a.a_sh = p->sh;
    UB_REQUIRE(kh_taps * kw_taps <= MAXT);
    // Up to three consecutive taps of a kernel row share one A load when the
    // kernel groups sub-taps (bf16 modes, tiles up to 192 columns; mode 4, tiles
    // up to 128 columns) and their shifts stay within the 8 rows of headroom.
    const int nsub = (((mode == 1 || mode == 3) && block_n <= 192) || mode == 4) ? 3 : 1;
    for (int i = 0; i < kh_taps; ++i)
      for (int j = 0; j < kw_taps;) {
        int n = kw_taps - j < nsub ? kw_taps - j : nsub;
        while (n > 1 && (n - 1) * p->dw > 8) --n;
        a.tap_dh[nt] = i * p->dh - p->ph;
        a.tap_dw[nt] = j * p->dw - p->pw;
        a.tap_c0[nt] = 0;
        a.tap_clen[nt] = p->c_in;
        a.tap_k0[nt] = (i * kw_taps + j) * p->c_in;
        a.tap_n[nt] = n;
        a.tap_k1[nt] = (i * kw_taps + j + 1) * p->c_in;
        a.tap_k2[nt] = (i * kw_taps + j + 2) * p->c_in;
        a.tap_s1[nt] = p->dw;
        a.tap_s2[nt] = 2 * p->dw;
        if ((n - 1) * p->dw > max_shift) max_shift = (n - 1) * p->dw;
        j += n;
        ++nt;
      }
  } else {
    // Stride-4, kernel-8, pad-2 time convolution read as "super rows" of 4
    // consecutive input rows: output w needs super rows w-1 (last two input
    // rows), w (all four) and w+1 (first two). Input rows past the logical
    // length must be zero up to a multiple of 4.
    UB_REQUIRE(p->sw == 4 && p->kw == 8 && p->pw == 2 && p->kh == 1 && p->h_in == 1 && p->dw == 1);
    UB_REQUIRE(p->in_sb % (4 * p->c_in) == 0);
    const int C = p->c_in;
    UB_REQUIRE((2 * C) % 32 == 0);
    dims[0] = (cuuint64_t)(4 * C);
    dims[1] = (cuuint64_t)((p->w_in + 3) / 4);
    dims[2] = 1;
    dims[3] = (cuuint64_t)p->batch;
    strides[0] = (cuuint64_t)(4 * C) * 4;
    strides[1] = (cuuint64_t)p->in_sb * 4;
    strides[2] = (cuuint64_t)p->in_sb * 4;
    a.a_sh = 0;
    const int c0s[3] = {2 * C, 0, 0}, clen[3] = {2 * C, 4 * C, 2 * C}, k0s[3] = {0, 2 * C, 6 * C};
    for (int i = 0; i < 3; ++i) {
      a.tap_dh[nt] = 0;
      a.tap_dw[nt] = i - 1;
      a.tap_c0[nt] = c0s[i];
      a.tap_clen[nt] = clen[i];
      a.tap_k0[nt] = k0s[i];
      a.tap_n[nt] = 1;
      ++nt;
    }
  }
  a.ntaps = nt;
  const int kc = (mode == 0 && block_n == 256) ? ChunkK<256, 0>::value : 32;
  const CUtensorMapSwizzle kc_swizzle = kc == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  int nch = 0;
  for (int i = 0; i < nt; ++i) nch += (a.tap_clen[i] + kc - 1) / kc;
  a.nchunks = nch;
  // Rows of one tile: all 128 unless a row of W does not split into 128s
  // (e.g. 336 STFT frames = 3 x 112).
  int m_valid = 128;
  if (p->w_out % 128 != 0 && p->h_out > 1) {
    for (int mv = 128; mv >= 64; mv -= 8)
      if (p->w_out % mv == 0) {
        m_valid = mv;
        break;
      }
  }
  a.m_valid = m_valid;
  a.m_box = m_valid;
  a.a_rows = m_valid + max_shift;
  UB_REQUIRE(max_shift <= 8);
  a.tiles_w = (p->w_out + m_valid - 1) / m_valid;
  a.tiles_n = (p->n_out + block_n - 1) / block_n;
  cuuint32_t boxA[4] = {(cuuint32_t)kc, (cuuint32_t)a.a_rows, 1, 1};
  if (mode == 3) {
    // bf16 rows of 32 channels (64 bytes): the MMA's 64-byte swizzled K-major layout.
    if (!make_map(&ma, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, x, dims, strides, boxA, CU_TENSOR_MAP_SWIZZLE_64B))
      return UNBLEND_ERR_INVALID;
  } else if (!make_map(&ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, x, dims, strides, boxA, kc_swizzle)) {
    return UNBLEND_ERR_INVALID;
  }
  // Weights [N, K] (K contiguous): fp32 hi/lo pair or bf16.
  cuuint64_t wd[2] = {(cuuint64_t)K, (cuuint64_t)p->n_out};
  if (mode == 0) {
    cuuint64_t ws[1] = {(cuuint64_t)K * 4};
    cuuint32_t boxB[2] = {(cuuint32_t)kc, (cuuint32_t)block_n};
    UB_REQUIRE((K * 4) % 16 == 0);
    if (!make_map(&mb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, w_hi, wd, ws, boxB, kc_swizzle) ||
        !make_map(&mb2, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, w_lo, wd, ws, boxB, kc_swizzle))
      return UNBLEND_ERR_INVALID;
  } else {
    cuuint64_t ws[1] = {(cuuint64_t)K * 2};
    cuuint32_t boxB[2] = {32, (cuuint32_t)block_n};
    UB_REQUIRE((K * 2) % 16 == 0);
    if (!make_map(&mb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w_hi, wd, ws, boxB, CU_TENSOR_MAP_SWIZZLE_64B))
      return UNBLEND_ERR_INVALID;
    mb2 = mb;
    if (bf16x3(mode) && !make_map(&mb2, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w_lo, wd, ws, boxB, CU_TENSOR_MAP_SWIZZLE_64B))
      return UNBLEND_ERR_INVALID;
  }
  const long long tiles = (long long)p->batch * p->h_out * a.tiles_w * a.tiles_n;
  UB_REQUIRE(tiles > 0 && tiles < (1LL << 31));
  a.tiles = tiles;
  // Output map for the bulk-store epilogue: (channel, w, h, b) with boxes of one
  // 16-row half of a warp's 32 positions x 32 channels (16 after GLU).
  CUtensorMap mo;
  memset(&mo, 0, sizeof(mo));
  const int n_final = p->act == UNBLEND_ACT_GLU ? p->n_out / 2 : p->n_out;
  a.tma_store = 0;
  // Stores go out in 16-row halves, so a tile's valid rows must be whole halves.
  if (!p->res && p->n_group >= n_final && p->out_sw >= n_final && m_valid % 16 == 0) {
    const int nv = p->act == UNBLEND_ACT_GLU ? 16 : 32;
    const int es = a.y_bf16 ? 2 : 4;  // output element bytes
    cuuint64_t od[4] = {(cuuint64_t)n_final, (cuuint64_t)p->w_out, (cuuint64_t)p->h_out, (cuuint64_t)p->batch};
    cuuint64_t os[3] = {(cuuint64_t)p->out_sw * es, (cuuint64_t)(p->out_sh > 0 ? p->out_sh : p->out_sw) * es,
                        (cuuint64_t)(p->out_sb > 0 ? p->out_sb : p->out_sw) * es};
    cuuint32_t ob[4] = {(cuuint32_t)nv, 16, 1, 1};
    if (make_map(&mo, a.y_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, y, od, os,
                 ob, nv * es == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B))
      a.tma_store = 1;
  }
  UB_REQUIRE(!a.y_bf16 || a.tma_store);  // bf16 output only leaves through the bulk stores
  cudaStream_t st = ub::as_stream(stream);
  if (mode == 0) {
    if (block_n == 64) return launch<64, 0>(ma, mb, mb2, mo, a, tiles, st);
    if (block_n == 96) return launch<96, 0>(ma, mb, mb2, mo, a, tiles, st);
    if (block_n == 128) return launch<128, 0>(ma, mb, mb2, mo, a, tiles, st);
    if (block_n == 192) return launch<192, 0>(ma, mb, mb2, mo, a, tiles, st);
    return launch<256, 0>(ma, mb, mb2, mo, a, tiles, st);
  }
  if (mode == 3) {
    if (block_n == 64) return launch<64, 3>(ma, mb, mb2, mo, a, tiles, st);
    if (block_n == 96) return launch<96, 3>(ma, mb, mb2, mo, a, tiles, st);
    if (block_n == 128) return launch<128, 3>(ma, mb, mb2, mo, a, tiles, st);
    if (block_n == 192) return launch<192, 3>(ma, mb, mb2, mo, a, tiles, st);
    return launch<256, 3>(ma, mb, mb2, mo, a, tiles, st);
  }
  if (mode == 4) {
    if (block_n == 64) return launch<64, 4>(ma, mb, mb2, mo, a, tiles, st);
    if (block_n == 96) return launch<96, 4>(ma, mb, mb2, mo, a, tiles, st);
    return launch<128, 4>(ma, mb, mb2, mo, a, tiles, st);
  }
  if (mode == 2) {
    if (block_n == 64) return launch<64, 2>(ma, mb, mb2, mo, a, tiles, st);
    if (block_n == 96) return launch<96, 2>(ma, mb, mb2, mo, a, tiles, st);
    if (block_n == 128) return launch<128, 2>(ma, mb, mb2, mo, a, tiles, st);
    if (block_n == 192) return launch<192, 2>(ma, mb, mb2, mo, a, tiles, st);
    return launch<256, 2>(ma, mb, mb2, mo, a, tiles, st);
  }
  if (block_n == 64) return launch<64, 1>(ma, mb, mb2, mo, a, tiles, st);
  if (block_n == 96) return launch<96, 1>(ma, mb, mb2, mo, a, tiles, st);
  if (block_n == 128) return launch<128, 1>(ma, mb, mb2, mo, a, tiles, st);
  if (block_n == 192) return launch<192, 1>(ma, mb, mb2, mo, a, tiles, st);
  return launch<256, 1>(ma, mb, mb2, mo, a, tiles, st);
}
