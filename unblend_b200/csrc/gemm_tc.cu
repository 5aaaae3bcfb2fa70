// Grouped linear layers on the tcgen05 tensor cores: a persistent kernel with
// a TMA producer, a single-thread MMA issuer and a double-buffered TMEM
// accumulator, so the epilogue of one 128 x BN tile overlaps the main loop of
// the next.
//
// Every group g computes out[r, out_col0 + j'] = epi(sum_k A[r, a_col0 + k] *
// W[w_row0 + j, k] + bias[w_row0 + j]) for all rows r of A (the M dimension,
// shared by the groups), j < n, k < kchunks * KC. One group is a plain
// nn.Linear over a token matrix; several groups express the per-band linears
// of BS-RoFormer's BandSplit and MaskEstimator (unblend/roformer.py:673-800)
// with one launch, each band reading its own column slice of A and its own
// block of weight rows. Weights beyond a group's true K are zero, so the K
// chunks may run into the next band's columns of A.
//
// Warp roles:
//   warp 0      TMA producer (one elected lane): A box [128 rows x KC], W box [BN rows x KC]
//   warp 1      TMEM allocation + MMA issue (one elected lane)
//   warps 2-9   epilogue: warp w reads TMEM lanes 32*(w%4).. (its 32 rows) for one half
//               of the tile's columns, 32 columns at a time; the 32x32 block is
//               transposed through a swizzled shared-memory tile so that each
//               lane then owns 4 consecutive columns of a row: bias loads are one
//               float4 per lane, and every global store / residual load of the
//               warp covers 4 whole row segments (coalesced)
//   warps 10-13 (MODE 0 only) split each fp32 A tile into TF32 hi + lo in shared memory
// MODE 0: fp32 A and fp32 hi/lo weights, D += Ahi*Whi + Ahi*Wlo + Alo*Whi in
// kind::tf32 (fp32-level accuracy). MODE 1: bf16 A and bf16 weights straight
// from TMA into kind::f16 MMAs (no conversion pass).
#include <cuda_bf16.h>
#include <cudaTypedefs.h>
#include <string.h>

#include "common.cuh"
#include "tc_common.cuh"

namespace {

using namespace ub::tc;

struct GroupDesc {
  int a_col0, w_row0, n, kchunks, out_col0, tile0, n_tiles;
};

struct GemmArgs {
  int m, groups, total_tiles;
  int act;
  int out_bf16;
  int vec;  // 1: all output / residual column runs are 16-byte aligned
  const float* bias;
  void* out;
  long long ldo;
  const float* res;
  long long ldr;
  const float2* rope;
  int rope_cols, rope_hd, rope_div, rope_mod;
  int tma_store;  // 1: whole 32-column chunks leave through TMA bulk stores (no residual)
  GroupDesc g[UNBLEND_GEMM_MAX_GROUPS];
};

constexpr int EPI_WARPS = 8;
constexpr int EPI_W0 = 2;                // first epilogue warp
constexpr int CONV_W0 = EPI_W0 + EPI_WARPS;
constexpr int EPI_TILE = 32 * 32 * 4;    // per-warp transpose tile (32 rows x 32 fp32)

template <int BN, int MODE>
struct GL {
  static constexpr int KC = MODE == 0 ? 32 : 64;  // K elements per stage (128-byte rows)
  static constexpr int A_BYTES = 128 * 128;
  static constexpr int ALO_BYTES = MODE == 0 ? 128 * 128 : 0;
  static constexpr int B_BYTES = BN * 128;
  static constexpr int B_TILES = MODE == 0 ? 2 : 1;
  static constexpr int STAGE = A_BYTES + ALO_BYTES + B_TILES * B_BYTES;
  static constexpr int EPI_BYTES = EPI_WARPS * EPI_TILE;
  static constexpr int STAGES_FIT = (227 * 1024 - EPI_BYTES - 1024 - 256) / STAGE;
  static constexpr int STAGES = STAGES_FIT > 6 ? 6 : STAGES_FIT;
  static constexpr int SMEM = STAGES * STAGE + EPI_BYTES + 1024 + 256;
  static constexpr int NT = 32 * (CONV_W0 + (MODE == 0 ? 4 : 0));
  static constexpr int TMEM_COLS = 2 * BN;
  static_assert(STAGES >= 2, "pipeline needs two stages");
};

// Tile t -> (group g, first row m0, n-tile index nt). Tiles are numbered group
// by group, and within a group n-tile fastest, so the CTAs running at one time
// share their A row blocks in L2.
__device__ __forceinline__ void decode_tile(const GemmArgs& a, int t, int& g, int& m0, int& nt) {
  g = 0;
  while (g + 1 < a.groups && t >= a.g[g + 1].tile0) ++g;
  const int local = t - a.g[g].tile0;
  const int n_tiles = a.g[g].n_tiles;
  m0 = (local / n_tiles) * 128;
  nt = local % n_tiles;
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map), "r"(src),
               "r"(x), "r"(y)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until every committed bulk store of this thread has finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Epilogue activation. FAST (the bf16 path, whose outputs are rounded to bf16
// or feed bf16 operands) uses the hardware tanh.approx instruction: tanh
// directly, and GELU in its tanh form 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715
// x^3))) (Hendrycks & Gimpel 2016), whose deviation from the exact erf GELU
// (< 5e-4 absolute) is below half a bf16 ulp of the result. The fp32 path keeps
// the exact erf GELU and tanhf.
template <int ACT, bool FAST>
__device__ __forceinline__ float act_fn(float x) {
  if (ACT == UNBLEND_ACT_GELU) {
    if (FAST) {
      const float z = 0.7978845608028654f * fmaf(0.044715f * x, x * x, x);
      return 0.5f * x * (1.0f + tanh_approx(z));
    }
    return ub::gelu_erf(x);
  }
  if (ACT == UNBLEND_ACT_TANH) return FAST ? tanh_approx(x) : tanhf(x);
  return x;
}

template <bool FAST>
__device__ __forceinline__ float sigmoid_fn(float x) {
  if (FAST) return 0.5f * tanh_approx(0.5f * x) + 0.5f;
  return ub::sigmoid_approx(x);
}

// Store NV (4, or 2 after GLU) consecutive values of one row at element
// offset `off` (cnt of them valid), adding the residual values `r` (already
// loaded by the caller) when present.
template <int NV, int OBF>
__device__ __forceinline__ void store_vals(const GemmArgs& a, long long off, float (&o)[NV], const float4& r,
                                           int cnt) {
  if (a.vec && cnt == NV) {
    if (a.res) {
      o[0] += r.x;
      o[1] += r.y;
      if (NV == 4) {
        o[2] += r.z;
        o[3] += r.w;
      }
    }
    if (OBF) {
      __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.out) + off;
      __nv_bfloat162 p0 = __floats2bfloat162_rn(o[0], o[1]);
      if (NV == 4) {
        __nv_bfloat162 p1 = __floats2bfloat162_rn(o[2], o[3]);
        uint2 packed;
        packed.x = *reinterpret_cast<uint32_t*>(&p0);
        packed.y = *reinterpret_cast<uint32_t*>(&p1);
        *reinterpret_cast<uint2*>(out) = packed;
      } else {
        *reinterpret_cast<__nv_bfloat162*>(out) = p0;
      }
    } else {
      float* out = reinterpret_cast<float*>(a.out) + off;
      if (NV == 4)
        *reinterpret_cast<float4*>(out) = make_float4(o[0], o[1], o[2], o[3]);
      else
        *reinterpret_cast<float2*>(out) = make_float2(o[0], o[1]);
    }
    return;
  }
  const float rr[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
  for (int e = 0; e < NV; ++e) {
    if (e < cnt) {
      float v = o[e];
      if (a.res) v += rr[e];
      if (OBF)
        reinterpret_cast<__nv_bfloat16*>(a.out)[off + e] = __float2bfloat16_rn(v);
      else
        reinterpret_cast<float*>(a.out)[off + e] = v;
    }
  }
}

template <int BN, int MODE, int ACT, int OBF>
__global__ void __launch_bounds__(GL<BN, MODE>::NT, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
                   const __grid_constant__ CUtensorMap mapB2, const __grid_constant__ CUtensorMap mapO,
                   const __grid_constant__ GemmArgs a) {
  using L = GL<BN, MODE>;
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
  if (warp == 1) tmem_alloc(tmem_slot, L::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < a.total_tiles && ok; t += gridDim.x) {
        int g, m0, nt;
        decode_tile(a, t, g, m0, nt);
        const GroupDesc& gd = a.g[g];
        const int n0 = nt * BN;
        for (int kc = 0; kc < gd.kchunks; ++kc, ++it) {
          const int s = it % L::STAGES;
          const int r = it / L::STAGES;
          if (r > 0 && !mbar_wait(&empty[s], (r - 1) & 1)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * L::STAGE;
          mbar_expect_tx(&full[s], (uint32_t)(L::A_BYTES + L::B_TILES * L::B_BYTES));
          tma_load_2d(st, &mapA, &full[s], gd.a_col0 + kc * L::KC, m0);
          uint8_t* sb = st + L::A_BYTES + L::ALO_BYTES;
          tma_load_2d(sb, &mapB, &full[s], kc * L::KC, gd.w_row0 + n0);
          if (MODE == 0) tma_load_2d(sb + L::B_BYTES, &mapB2, &full[s], kc * L::KC, gd.w_row0 + n0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc(MODE == 0 ? 2u : 1u, (uint32_t)BN);
      int it = 0, i = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < a.total_tiles && ok; t += gridDim.x, ++i) {
        int g, m0, nt;
        decode_tile(a, t, g, m0, nt);
        const int kch = a.g[g].kchunks;
        const int buf = i & 1, u = i >> 1;
        if (u > 0 && !mbar_wait(&acc_empty[buf], (u - 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * BN);
        for (int kc = 0; kc < kch; ++kc, ++it) {
          const int s = it % L::STAGES;
          const int r = it / L::STAGES;
          if (!mbar_wait(MODE == 0 ? &conv[s] : &full[s], r & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * L::STAGE);
          const uint32_t sal = sa + L::A_BYTES;
          const uint32_t sb = sa + L::A_BYTES + L::ALO_BYTES;
          if (MODE == 0) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint64_t dah = smem_desc(sa + 32 * j, 128), dal = smem_desc(sal + 32 * j, 128);
              const uint64_t dbh = smem_desc(sb + 32 * j, 128), dbl = smem_desc(sb + L::B_BYTES + 32 * j, 128);
              umma_tf32(d, dah, dbh, idesc, (kc > 0 || j > 0) ? 1u : 0u);
              umma_tf32(d, dah, dbl, idesc, 1u);
              umma_tf32(d, dal, dbh, idesc, 1u);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 4; ++j)
              umma_bf16(d, smem_desc(sa + 32 * j, 128), smem_desc(sb + 32 * j, 128), idesc,
                        (kc > 0 || j > 0) ? 1u : 0u);
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&acc_full[buf]);
      }
      if (!ok) atomicExch(&g_error_flag, 2);
    }
  } else if (warp < CONV_W0) {
    // Epilogue warps.
    const int e = warp - EPI_W0;
    const int q = warp & 3;           // TMEM lane quarter this warp may read
    const int c_lo = (e >> 2) * (BN / 2);
    float4* stage = reinterpret_cast<float4*>(epi_smem + e * EPI_TILE);
    const int ch = lane & 7;          // this lane's 4-column group after the transpose
    int i = 0;
    for (int t = blockIdx.x; t < a.total_tiles; t += gridDim.x, ++i) {
      int g, m0, nt;
      decode_tile(a, t, g, m0, nt);
      const GroupDesc& gd = a.g[g];
      const int n0 = nt * BN;
      const int buf = i & 1, u = i >> 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[buf], u & 1))) break;
      tc_fence_after();
      const long long row0 = (long long)m0 + q * 32;
      const uint32_t base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN);
      // Rotary position of this lane's own TMEM row (the TMA-store path keeps lane = row).
      const int my_row = (int)row0 + lane;
      const int rope_pos = a.rope ? (my_row / a.rope_div) % a.rope_mod : 0;
#pragma unroll 1
      for (int c0 = c_lo; c0 < c_lo + BN / 2; c0 += 32) {
        if (n0 + c0 >= gd.n) break;  // uniform across the warp
        const bool bulk = a.tma_store && n0 + c0 + 32 <= gd.n;
        // Residual row segment of this lane (lane = row on the bulk path), loaded
        // before the TMEM read so the two latencies overlap.
        float4 rr[8];
        if (ACT != UNBLEND_ACT_GLU && bulk && a.res) {
          const float4* rp = reinterpret_cast<const float4*>(a.res + (long long)my_row * a.ldr + gd.out_col0 + n0 + c0);
#pragma unroll
          for (int j = 0; j < 8; ++j) rr[j] = my_row < a.m ? rp[j] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        uint32_t acc[32];
        tmem_ld32(base + (uint32_t)c0, acc);
        if (bulk) {
          // Whole chunk: activation in the lane = row layout, packed into a
          // swizzled staging tile, stored by one bulk tensor copy.
          constexpr bool FAST = MODE == 1;
          constexpr int NV = ACT == UNBLEND_ACT_GLU ? 16 : 32;      // values per row
          constexpr int RB = NV * (OBF ? 2 : 4);                     // staging row bytes: 32, 64 or 128
          constexpr int CH = RB / 16;                                // 16-byte chunks per row
          float v[32];
          if (a.bias) {
            const float4* bp = reinterpret_cast<const float4*>(a.bias + gd.w_row0 + n0 + c0);
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
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = act_fn<ACT, FAST>(v[j]);
          if (ACT == UNBLEND_ACT_NONE && a.rope && n0 + c0 < a.rope_cols) {
            const float4* cs = reinterpret_cast<const float4*>(a.rope + (long long)rope_pos * (a.rope_hd >> 1) +
                                                                (((n0 + c0) % a.rope_hd) >> 1));
#pragma unroll
            for (int j = 0; j < 8; ++j) {  // pairs (4j, 4j+1) and (4j+2, 4j+3)
              const float4 c2 = __ldg(cs + j);
              const float x0 = v[4 * j], x1 = v[4 * j + 1], x2 = v[4 * j + 2], x3 = v[4 * j + 3];
              v[4 * j] = x0 * c2.x - x1 * c2.y;
              v[4 * j + 1] = x0 * c2.y + x1 * c2.x;
              v[4 * j + 2] = x2 * c2.z - x3 * c2.w;
              v[4 * j + 3] = x2 * c2.w + x3 * c2.z;
            }
          }
          if (ACT != UNBLEND_ACT_GLU && a.res) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              v[4 * j] += rr[j].x;
              v[4 * j + 1] += rr[j].y;
              v[4 * j + 2] += rr[j].z;
              v[4 * j + 3] += rr[j].w;
            }
          }
          uint32_t w[OBF ? NV / 2 : NV];  // the packed row: NV/2 words of bf16 pairs, or NV fp32 words
#pragma unroll
          for (int j = 0; j < NV; ++j) {
            const float o = ACT == UNBLEND_ACT_GLU ? v[2 * j] * sigmoid_fn<FAST>(v[2 * j + 1]) : v[j];
            if (OBF) {
              if (j & 1) {
                __nv_bfloat162 b2 = __floats2bfloat162_rn(__uint_as_float(w[j >> 1]), o);
                w[j >> 1] = *reinterpret_cast<uint32_t*>(&b2);
              } else {
                w[j >> 1] = __float_as_uint(o);
              }
            } else {
              w[j] = __float_as_uint(o);
            }
          }
          uint8_t* stg = epi_smem + e * EPI_TILE;
          if (lane == 0) bulk_wait_read();  // the previous store has left the staging tile
          __syncwarp();
          const int swz = ((lane * RB) >> 7) & (CH - 1);
#pragma unroll
          for (int j = 0; j < CH; ++j)
            *reinterpret_cast<uint4*>(stg + lane * RB + ((j ^ swz) << 4)) =
                make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            const int x = gd.out_col0 + (ACT == UNBLEND_ACT_GLU ? (n0 + c0) / 2 : n0 + c0);
            tma_store_2d(&mapO, smem_u32(stg), x, (int)row0);
          }
          continue;
        }
        if (a.tma_store && lane == 0) bulk_wait_read();
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; ++j)
          stage[lane * 8 + (j ^ (lane & 7))] =
              make_float4(__uint_as_float(acc[4 * j]), __uint_as_float(acc[4 * j + 1]),
                          __uint_as_float(acc[4 * j + 2]), __uint_as_float(acc[4 * j + 3]));
        __syncwarp();
        const int ncol = n0 + c0 + ch * 4;  // group-local column of this lane's first value
        const int nvalid = min(4, gd.n - ncol);
        float4 bv = make_float4(0.f, 0.f, 0.f, 0.f);
        if (a.bias && nvalid > 0) {
          const float* bp = a.bias + gd.w_row0 + ncol;
          if (nvalid == 4) {
            bv = __ldg(reinterpret_cast<const float4*>(bp));
          } else {
            bv.x = __ldg(bp);
            if (nvalid > 1) bv.y = __ldg(bp + 1);
            if (nvalid > 2) bv.z = __ldg(bp + 2);
          }
        }
        constexpr bool FAST = MODE == 1;
        const int oc = gd.out_col0 + (ACT == UNBLEND_ACT_GLU ? ncol / 2 : ncol);
        const int ocnt = ACT == UNBLEND_ACT_GLU ? nvalid / 2 : nvalid;
        // Residual values of the lane's 8 rows, all loads in flight at once.
        float4 rv[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          rv[k] = make_float4(0.f, 0.f, 0.f, 0.f);
          const long long row = row0 + k * 4 + (lane >> 3);
          if (a.res && row < a.m && nvalid > 0) {
            const float* rp = a.res + row * a.ldr + oc;
            if (a.vec && ocnt == (ACT == UNBLEND_ACT_GLU ? 2 : 4)) {
              if (ACT == UNBLEND_ACT_GLU) {
                const float2 t2 = *reinterpret_cast<const float2*>(rp);
                rv[k] = make_float4(t2.x, t2.y, 0.f, 0.f);
              } else {
                rv[k] = *reinterpret_cast<const float4*>(rp);
              }
            } else {
              rv[k].x = rp[0];
              if (ocnt > 1) rv[k].y = rp[1];
              if (ocnt > 2) rv[k].z = rp[2];
              if (ocnt > 3) rv[k].w = rp[3];
            }
          }
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int r = k * 4 + (lane >> 3);
          const long long row = row0 + r;
          const float4 v = stage[r * 8 + (ch ^ (r & 7))];
          if (row >= a.m || nvalid <= 0) continue;
          float x[4] = {act_fn<ACT, FAST>(v.x + bv.x), act_fn<ACT, FAST>(v.y + bv.y),
                        act_fn<ACT, FAST>(v.z + bv.z), act_fn<ACT, FAST>(v.w + bv.w)};
          if (ACT == UNBLEND_ACT_NONE && a.rope && ncol < a.rope_cols) {
            const int pos = ((int)row / a.rope_div) % a.rope_mod;  // rows < 2^31 (checked on the host)
            const float2* cs = a.rope + (long long)pos * (a.rope_hd >> 1) + ((ncol % a.rope_hd) >> 1);
            const float2 c0 = __ldg(cs), c1 = __ldg(cs + 1);
            const float x0 = x[0], x1 = x[1], x2 = x[2], x3 = x[3];
            x[0] = x0 * c0.x - x1 * c0.y;
            x[1] = x0 * c0.y + x1 * c0.x;
            x[2] = x2 * c1.x - x3 * c1.y;
            x[3] = x2 * c1.y + x3 * c1.x;
          }
          if (ACT == UNBLEND_ACT_GLU) {
            float o[2] = {x[0] * sigmoid_fn<FAST>(x[1]), x[2] * sigmoid_fn<FAST>(x[3])};
            store_vals<2, OBF>(a, row * a.ldo + oc, o, rv[k], ocnt);
          } else {
            store_vals<4, OBF>(a, row * a.ldo + oc, x, rv[k], ocnt);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
    if (a.tma_store && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    __syncwarp();
  } else if (MODE == 0) {
    // Converter warps: TF32 hi (in place) + lo split of each fp32 A tile.
    const int ct = threadIdx.x - 32 * CONV_W0;
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < a.total_tiles && ok; t += gridDim.x) {
      int g, m0, nt;
      decode_tile(a, t, g, m0, nt);
      const int kch = a.g[g].kchunks;
      for (int kc = 0; kc < kch; ++kc, ++it) {
        const int s = it % L::STAGES;
        const int r = it / L::STAGES;
        if (!mbar_wait(&full[s], r & 1)) {
          ok = false;
          break;
        }
        uint8_t* st = smem + s * L::STAGE;
        float4* hi = reinterpret_cast<float4*>(st);
        float4* lo = reinterpret_cast<float4*>(st + L::A_BYTES);
#pragma unroll
        for (int k = ct; k < 1024; k += 128) {
          const float4 v = hi[k];
          float4 vh;
          vh.x = __uint_as_float((__float_as_uint(v.x) + 0x1000u) & 0xFFFFE000u);
          vh.y = __uint_as_float((__float_as_uint(v.y) + 0x1000u) & 0xFFFFE000u);
          vh.z = __uint_as_float((__float_as_uint(v.z) + 0x1000u) & 0xFFFFE000u);
          vh.w = __uint_as_float((__float_as_uint(v.w) + 0x1000u) & 0xFFFFE000u);
          hi[k] = vh;
          lo[k] = make_float4(v.x - vh.x, v.y - vh.y, v.z - vh.z, v.w - vh.w);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[s]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
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

// 2-D K-major map (cols contiguous, rows at `row_bytes`) with a box of
// [box_rows x 128 bytes] and the 128-byte swizzle.
bool map_2d(CUtensorMap* m, bool bf16, const void* base, long long cols, long long rows, long long row_bytes,
            int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  const int esz = bf16 ? 2 : 4;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  cuuint32_t box[2] = {(cuuint32_t)(128 / esz), (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  return fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base),
            dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ub::kNumSMs;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return ub::kNumSMs;
  return n;
}

template <int BN, int MODE, int ACT, int OBF>
int launch(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mb2, const CUtensorMap& mo,
           const GemmArgs& args, cudaStream_t st) {
  using L = GL<BN, MODE>;
  auto k = gemm_tc_kernel<BN, MODE, ACT, OBF>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM);
  int grid = sm_count();
  if (grid > args.total_tiles) grid = args.total_tiles;
  k<<<grid, L::NT, L::SMEM, st>>>(ma, mb, mb2, mo, args);
  UB_CHECK_LAUNCH();
  return 0;
}

template <int BN, int MODE>
int dispatch_epi(int act, int obf, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mb2,
                 const CUtensorMap& mo, const GemmArgs& g, cudaStream_t st) {
  switch (act * 2 + obf) {
    case UNBLEND_ACT_NONE * 2: return launch<BN, MODE, UNBLEND_ACT_NONE, 0>(ma, mb, mb2, mo, g, st);
    case UNBLEND_ACT_NONE * 2 + 1: return launch<BN, MODE, UNBLEND_ACT_NONE, 1>(ma, mb, mb2, mo, g, st);
    case UNBLEND_ACT_GELU * 2: return launch<BN, MODE, UNBLEND_ACT_GELU, 0>(ma, mb, mb2, mo, g, st);
    case UNBLEND_ACT_GELU * 2 + 1: return launch<BN, MODE, UNBLEND_ACT_GELU, 1>(ma, mb, mb2, mo, g, st);
    case UNBLEND_ACT_GLU * 2: return launch<BN, MODE, UNBLEND_ACT_GLU, 0>(ma, mb, mb2, mo, g, st);
    case UNBLEND_ACT_GLU * 2 + 1: return launch<BN, MODE, UNBLEND_ACT_GLU, 1>(ma, mb, mb2, mo, g, st);
    case UNBLEND_ACT_TANH * 2: return launch<BN, MODE, UNBLEND_ACT_TANH, 0>(ma, mb, mb2, mo, g, st);
    case UNBLEND_ACT_TANH * 2 + 1: return launch<BN, MODE, UNBLEND_ACT_TANH, 1>(ma, mb, mb2, mo, g, st);
    default: return UNBLEND_ERR_INVALID;
  }
}

int dispatch_mode(int mode, int block_n, int act, int obf, const CUtensorMap& ma, const CUtensorMap& mb,
                  const CUtensorMap& mb2, const CUtensorMap& mo, const GemmArgs& g, cudaStream_t st) {
  if (mode == 0) {
    if (block_n == 64) return dispatch_epi<64, 0>(act, obf, ma, mb, mb2, mo, g, st);
    if (block_n == 128) return dispatch_epi<128, 0>(act, obf, ma, mb, mb2, mo, g, st);
    return dispatch_epi<256, 0>(act, obf, ma, mb, mb2, mo, g, st);
  }
  if (block_n == 64) return dispatch_epi<64, 1>(act, obf, ma, mb, mb2, mo, g, st);
  if (block_n == 128) return dispatch_epi<128, 1>(act, obf, ma, mb, mb2, mo, g, st);
  return dispatch_epi<256, 1>(act, obf, ma, mb, mb2, mo, g, st);
}

}  // namespace

extern "C" int unblend_gemm_tc(const void* a, long long lda, int rows, int a_cols, const void* w_hi, const void* w_lo,
                               long long w_rows, int w_cols, const UnblendGemmParams* p, int mode, int block_n,
                               void* stream) {
  UB_REQUIRE(a && w_hi && p && p->out && rows > 0 && a_cols > 0 && w_rows > 0 && w_cols > 0);
  UB_REQUIRE(mode == 0 || mode == 1);
  UB_REQUIRE(mode == 1 || w_lo);
  UB_REQUIRE(block_n == 64 || block_n == 128 || block_n == 256);
  UB_REQUIRE(p->groups >= 1 && p->groups <= UNBLEND_GEMM_MAX_GROUPS && p->group);
  UB_REQUIRE(p->act == UNBLEND_ACT_NONE || p->act == UNBLEND_ACT_GELU || p->act == UNBLEND_ACT_GLU ||
             p->act == UNBLEND_ACT_TANH);
  const int esz = mode == 0 ? 4 : 2;
  const int kc = mode == 0 ? 32 : 64;
  const int align = 16 / esz;  // elements per 16 bytes
  UB_REQUIRE((reinterpret_cast<uintptr_t>(a) & 15) == 0 && (reinterpret_cast<uintptr_t>(w_hi) & 15) == 0);
  UB_REQUIRE(mode == 1 || (reinterpret_cast<uintptr_t>(w_lo) & 15) == 0);
  UB_REQUIRE(lda >= a_cols && lda % align == 0 && w_cols % align == 0);
  UB_REQUIRE(p->ldo > 0 && (!p->res || p->ldr > 0));
  UB_REQUIRE(!p->bias || (reinterpret_cast<uintptr_t>(p->bias) & 15) == 0);
  GemmArgs g{};
  g.m = rows;
  g.groups = p->groups;
  g.act = p->act;
  g.out_bf16 = p->out_bf16 ? 1 : 0;
  g.bias = p->bias;
  g.out = p->out;
  g.ldo = p->ldo;
  g.res = p->res;
  g.ldr = p->ldr;
  if (p->rope) {
    UB_REQUIRE(p->act == UNBLEND_ACT_NONE && p->rope_hd >= 4 && p->rope_hd % 4 == 0 && p->rope_cols % 4 == 0);
    UB_REQUIRE(p->rope_div > 0 && p->rope_mod > 0 && (reinterpret_cast<uintptr_t>(p->rope) & 7) == 0);
    g.rope = reinterpret_cast<const float2*>(p->rope);
    g.rope_cols = p->rope_cols;
    g.rope_hd = p->rope_hd;
    g.rope_div = p->rope_div;
    g.rope_mod = p->rope_mod;
  }
  const int m_tiles = (rows + 127) / 128;  // rows is an int: row indices fit 32 bits
  long long tiles = 0;
  bool vec = (reinterpret_cast<uintptr_t>(p->out) & 15) == 0 && p->ldo % 4 == 0;
  if (p->res) vec = vec && (reinterpret_cast<uintptr_t>(p->res) & 15) == 0 && p->ldr % 4 == 0;
  for (int i = 0; i < p->groups; ++i) {
    const UnblendGemmGroup& s = p->group[i];
    UB_REQUIRE(s.n > 0 && s.k > 0 && s.k <= w_cols && s.a_col0 >= 0 && s.a_col0 % align == 0 && s.a_col0 < a_cols);
    UB_REQUIRE(s.w_row0 >= 0 && s.w_row0 + (long long)s.n <= w_rows && s.out_col0 >= 0);
    UB_REQUIRE(p->act != UNBLEND_ACT_GLU || s.n % 4 == 0);
    UB_REQUIRE(!p->bias || s.w_row0 % 4 == 0);
    if (s.out_col0 % 4 != 0) vec = false;
    GroupDesc& d = g.g[i];
    d.a_col0 = s.a_col0;
    d.w_row0 = s.w_row0;
    d.n = s.n;
    d.kchunks = (s.k + kc - 1) / kc;
    d.out_col0 = s.out_col0;
    d.tile0 = (int)tiles;
    d.n_tiles = (s.n + block_n - 1) / block_n;
    tiles += (long long)m_tiles * d.n_tiles;
  }
  UB_REQUIRE(tiles > 0 && tiles < (1LL << 31));
  g.total_tiles = (int)tiles;
  g.vec = vec ? 1 : 0;
  CUtensorMap ma, mb, mb2;
  if (!map_2d(&ma, mode == 1, a, a_cols, rows, lda * esz, 128)) return UNBLEND_ERR_INVALID;
  if (!map_2d(&mb, mode == 1, w_hi, w_cols, w_rows, (long long)w_cols * esz, block_n)) return UNBLEND_ERR_INVALID;
  if (mode == 0) {
    if (!map_2d(&mb2, false, w_lo, w_cols, w_rows, (long long)w_cols * 4, block_n)) return UNBLEND_ERR_INVALID;
  } else {
    mb2 = mb;
  }
  // Output tensor map for the bulk-store epilogue: [rows, ldo] with a box of one
  // 32-row chunk (32 columns, 16 after GLU) and the swizzle matching its row bytes.
  CUtensorMap mo;
  memset(&mo, 0, sizeof(mo));
  const int oesz = g.out_bf16 ? 2 : 4;
  // Residual epilogues keep the transposed path (prefetched residual rows):
  // measured faster than per-lane residual reads on the bulk path.
  bool tma = !p->res && (reinterpret_cast<uintptr_t>(p->out) & 15) == 0 && (p->ldo * oesz) % 16 == 0;
  for (int i = 0; i < p->groups && tma; ++i) tma = (p->group[i].out_col0 * oesz) % 16 == 0;
  if (tma) {
    const int nv = p->act == UNBLEND_ACT_GLU ? 16 : 32;
    const int rb = nv * oesz;
    const CUtensorMapSwizzle sw = rb == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                  : rb == 64  ? CU_TENSOR_MAP_SWIZZLE_64B
                                              : CU_TENSOR_MAP_SWIZZLE_32B;
    cuuint64_t dims[2] = {(cuuint64_t)p->ldo, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)p->ldo * oesz};
    cuuint32_t box[2] = {(cuuint32_t)nv, 32};
    cuuint32_t es[2] = {1, 1};
    auto fn = encode_fn();
    tma = fn && fn(&mo, g.out_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, p->out,
                   dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  }
  g.tma_store = tma ? 1 : 0;
  return dispatch_mode(mode, block_n, p->act, g.out_bf16, ma, mb, mb2, mo, g, ub::as_stream(stream));
}

extern "C" int unblend_gemm_error_flag(int* out_host, int clear) {
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
