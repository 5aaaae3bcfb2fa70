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
//   warps 2-5   epilogue: TMEM -> registers -> bias / activation / residual -> global
//   warps 6-9   (MODE 0 only) split each fp32 A tile into TF32 hi + lo in shared memory
// MODE 0: fp32 A and fp32 hi/lo weights, D += Ahi*Whi + Ahi*Wlo + Alo*Whi in
// kind::tf32 (fp32-level accuracy). MODE 1: bf16 A and bf16 weights straight
// from TMA into kind::f16 MMAs (no conversion pass).
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

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
  GroupDesc g[UNBLEND_GEMM_MAX_GROUPS];
};

template <int BN, int MODE>
struct GL {
  static constexpr int KC = MODE == 0 ? 32 : 64;  // K elements per stage (128-byte rows)
  static constexpr int A_BYTES = 128 * 128;
  static constexpr int ALO_BYTES = MODE == 0 ? 128 * 128 : 0;
  static constexpr int B_BYTES = BN * 128;
  static constexpr int B_TILES = MODE == 0 ? 2 : 1;
  static constexpr int STAGE = A_BYTES + ALO_BYTES + B_TILES * B_BYTES;
  static constexpr int STAGES_FIT = (200 * 1024) / STAGE;
  static constexpr int STAGES = STAGES_FIT > 6 ? 6 : STAGES_FIT;
  static constexpr int SMEM = STAGES * STAGE + 1024 + 256;
  static constexpr int NT = MODE == 0 ? 320 : 192;
  static constexpr int TMEM_COLS = 2 * BN;
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

__device__ __forceinline__ float act_fn(float x, int act) {
  if (act == UNBLEND_ACT_GELU) return ub::gelu_erf(x);
  if (act == UNBLEND_ACT_TANH) return tanhf(x);
  return x;
}

// Store `cnt` (<= NOUT) values o[0..cnt) at column `col` of row `row`, adding
// the residual first when present.
template <int NOUT>
__device__ __forceinline__ void store_run(const GemmArgs& a, long long row, int col, float (&o)[NOUT], int cnt) {
  const long long ro = row * a.ldr + col;
  const long long oo = row * a.ldo + col;
#pragma unroll
  for (int j4 = 0; j4 < NOUT / 4; ++j4) {
    if (4 * j4 >= cnt) break;
    if (a.vec && 4 * j4 + 4 <= cnt) {
      float v0 = o[4 * j4], v1 = o[4 * j4 + 1], v2 = o[4 * j4 + 2], v3 = o[4 * j4 + 3];
      if (a.res) {
        const float4 r = *reinterpret_cast<const float4*>(a.res + ro + 4 * j4);
        v0 += r.x;
        v1 += r.y;
        v2 += r.z;
        v3 += r.w;
      }
      if (a.out_bf16) {
        __nv_bfloat162 p0 = __floats2bfloat162_rn(v0, v1);
        __nv_bfloat162 p1 = __floats2bfloat162_rn(v2, v3);
        uint2 packed;
        packed.x = *reinterpret_cast<uint32_t*>(&p0);
        packed.y = *reinterpret_cast<uint32_t*>(&p1);
        *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(a.out) + oo + 4 * j4) = packed;
      } else {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(a.out) + oo + 4 * j4) = make_float4(v0, v1, v2, v3);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (4 * j4 + e < cnt) {
          float v = o[4 * j4 + e];
          if (a.res) v += a.res[ro + 4 * j4 + e];
          if (a.out_bf16)
            reinterpret_cast<__nv_bfloat16*>(a.out)[oo + 4 * j4 + e] = __float2bfloat16_rn(v);
          else
            reinterpret_cast<float*>(a.out)[oo + 4 * j4 + e] = v;
        }
      }
    }
  }
}

template <int BN, int MODE>
__global__ void __launch_bounds__(GL<BN, MODE>::NT, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
                   const __grid_constant__ CUtensorMap mapB2, const __grid_constant__ GemmArgs a) {
  using L = GL<BN, MODE>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::STAGES * L::STAGE);
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
      mbar_init(&acc_empty[i], 4);
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
  } else if (warp < 6) {
    // Epilogue warps: warp w reads TMEM lanes 32*(w%4) .. 32*(w%4)+31.
    const int q = warp & 3;
    int i = 0;
    for (int t = blockIdx.x; t < a.total_tiles; t += gridDim.x, ++i) {
      int g, m0, nt;
      decode_tile(a, t, g, m0, nt);
      const GroupDesc& gd = a.g[g];
      const int n0 = nt * BN;
      const int buf = i & 1, u = i >> 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[buf], u & 1))) break;
      tc_fence_after();
      const long long row = (long long)m0 + q * 32 + lane;
      const bool rv = row < a.m;
      const uint32_t base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN);
      const bool glu = a.act == UNBLEND_ACT_GLU;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        if (n0 + c0 >= gd.n) break;  // uniform across the warp
        uint32_t acc[32];
        __syncwarp();
        tmem_ld32(base + (uint32_t)c0, acc);
        if (!rv) continue;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int n = n0 + c0 + j;
          float x = __uint_as_float(acc[j]);
          if (a.bias && n < gd.n) x += __ldg(a.bias + gd.w_row0 + n);
          v[j] = act_fn(x, a.act);
        }
        if (glu) {
          float o[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) o[j] = v[2 * j] * ub::sigmoidf_(v[2 * j + 1]);
          const int col = (n0 + c0) / 2;
          const int cnt = min(16, gd.n / 2 - col);
          store_run<16>(a, row, gd.out_col0 + col, o, cnt);
        } else {
          const int col = n0 + c0;
          const int cnt = min(32, gd.n - col);
          store_run<32>(a, row, gd.out_col0 + col, v, cnt);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  } else if (MODE == 0) {
    // Converter warps 6-9: TF32 hi (in place) + lo split of each fp32 A tile.
    const int ct = threadIdx.x - 192;
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

template <int BN, int MODE>
int launch(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mb2, const GemmArgs& args,
           cudaStream_t st) {
  using L = GL<BN, MODE>;
  auto k = gemm_tc_kernel<BN, MODE>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM);
  int grid = sm_count();
  if (grid > args.total_tiles) grid = args.total_tiles;
  k<<<grid, L::NT, L::SMEM, st>>>(ma, mb, mb2, args);
  UB_CHECK_LAUNCH();
  return 0;
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
  const int m_tiles = (rows + 127) / 128;
  long long tiles = 0;
  bool vec = (reinterpret_cast<uintptr_t>(p->out) & 15) == 0 && p->ldo % 4 == 0;
  if (p->res) vec = vec && (reinterpret_cast<uintptr_t>(p->res) & 15) == 0 && p->ldr % 4 == 0;
  for (int i = 0; i < p->groups; ++i) {
    const UnblendGemmGroup& s = p->group[i];
    UB_REQUIRE(s.n > 0 && s.k > 0 && s.k <= w_cols && s.a_col0 >= 0 && s.a_col0 % align == 0 && s.a_col0 < a_cols);
    UB_REQUIRE(s.w_row0 >= 0 && s.w_row0 + (long long)s.n <= w_rows && s.out_col0 >= 0);
    UB_REQUIRE(p->act != UNBLEND_ACT_GLU || s.n % 2 == 0);
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
  cudaStream_t st = ub::as_stream(stream);
  if (mode == 0) {
    if (block_n == 64) return launch<64, 0>(ma, mb, mb2, g, st);
    if (block_n == 128) return launch<128, 0>(ma, mb, mb2, g, st);
    return launch<256, 0>(ma, mb, mb2, g, st);
  }
  if (block_n == 64) return launch<64, 1>(ma, mb, mb2, g, st);
  if (block_n == 128) return launch<128, 1>(ma, mb, mb2, g, st);
  return launch<256, 1>(ma, mb, mb2, g, st);
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
