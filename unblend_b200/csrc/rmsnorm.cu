// RMSNorm kernels of BS-RoFormer (unblend/roformer.py:60-91: F.rms_norm with
// eps 1e-12, y = x * rsqrt(mean(x^2) + eps) * gamma).
//
// rms_norm_kernel: one warp per token row (the pre-norms of Attention and
//   FeedForward, the final norm). Optionally also produces the attention
//   gates sigmoid(y . Wg[h] + bg[h]) of the gated Attention
//   (unblend/roformer.py:478-511) from the fp32 normalised row, so the row is
//   read once for both.
// band_rms_norm_kernel: one warp per (row, band): each band's slice of the
//   STFT feature row is normalised on its own (BandSplit,
//   unblend/roformer.py:673-705).
#include <cuda_bf16.h>

#include "common.cuh"

namespace {

constexpr float kEps = 1e-12f;
constexpr int kMaxVec = 8;    // float4s per lane: dim <= 1024
constexpr int kMaxGates = 16;

__device__ __forceinline__ void store4(void* y, long long off, float4 v, int bf16) {
  if (bf16) {
    __nv_bfloat162 p0 = __floats2bfloat162_rn(v.x, v.y);
    __nv_bfloat162 p1 = __floats2bfloat162_rn(v.z, v.w);
    uint2 packed;
    packed.x = *reinterpret_cast<uint32_t*>(&p0);
    packed.y = *reinterpret_cast<uint32_t*>(&p1);
    *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(y) + off) = packed;
  } else {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(y) + off) = v;
  }
}

// Sum each of v[0..15] over the warp; lane l ends up holding the total of
// v[idx(l)] with idx(l) = 8*b4 + 4*b3 + 2*b2 + b1 (b_k = bit k of l), in 16
// shuffles instead of 80 (a butterfly reduce-scatter).
__device__ __forceinline__ float reduce16(float (&v)[16], int lane) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const bool up = lane & 16;
    const float send = up ? v[i] : v[i + 8];
    const float keep = up ? v[i + 8] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const bool up = lane & 8;
    const float send = up ? v[i] : v[i + 4];
    const float keep = up ? v[i + 4] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const bool up = lane & 4;
    const float send = up ? v[i] : v[i + 2];
    const float keep = up ? v[i + 2] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  {
    const bool up = lane & 2;
    const float send = up ? v[0] : v[1];
    const float keep = up ? v[1] : v[0];
    v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
}

// One warp normalises ROWS rows per iteration (independent loads in flight);
// with gates, each gate weight read from shared memory serves all ROWS rows.
template <int ROWS>
__global__ void __launch_bounds__(256) rms_norm_kernel(const float* __restrict__ x, long long rows, int dim,
                                                       const float* __restrict__ gamma, void* __restrict__ y,
                                                       long long ldy, int y_bf16, const float* __restrict__ gw,
                                                       const float* __restrict__ gb, int gates,
                                                       float* __restrict__ gout) {
  extern __shared__ float s_gw[];  // [gates, dim]
  for (int i = threadIdx.x; i < gates * dim; i += blockDim.x) s_gw[i] = gw[i];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int nv = dim >> 2;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  const long long groups = (rows + ROWS - 1) / ROWS;
  for (long long gi = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5); gi < groups; gi += warps) {
    const long long r0 = gi * ROWS;
    float4 v[ROWS][kMaxVec];
    float inv[ROWS];
#pragma unroll
    for (int k = 0; k < ROWS; ++k) {
      const bool rv = r0 + k < rows;
      const float4* xr = reinterpret_cast<const float4*>(x + (r0 + k) * dim);
#pragma unroll
      for (int i = 0; i < kMaxVec; ++i) {
        const int c = lane + 32 * i;
        v[k][i] = rv && c < nv ? __ldg(xr + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int k = 0; k < ROWS; ++k) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < kMaxVec; ++i)
        ss += v[k][i].x * v[k][i].x + v[k][i].y * v[k][i].y + v[k][i].z * v[k][i].z + v[k][i].w * v[k][i].w;
      ss = ub::warp_sum(ss);
      inv[k] = rsqrtf(ss / (float)dim + kEps);
    }
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
      const int c = lane + 32 * i;
      if (c < nv) {
        const float4 g = __ldg(reinterpret_cast<const float4*>(gamma) + c);
#pragma unroll
        for (int k = 0; k < ROWS; ++k) {
          v[k][i] = make_float4(v[k][i].x * inv[k] * g.x, v[k][i].y * inv[k] * g.y, v[k][i].z * inv[k] * g.z,
                                v[k][i].w * inv[k] * g.w);
          if (r0 + k < rows) store4(y, (r0 + k) * ldy + 4 * c, v[k][i], y_bf16);
        }
      }
    }
    if (gates == 8 && ROWS == 2) {
      float acc[16];
#pragma unroll
      for (int q = 0; q < 16; ++q) acc[q] = 0.f;
#pragma unroll
      for (int i = 0; i < kMaxVec; ++i) {
        const int c = lane + 32 * i;
        if (c < nv) {
#pragma unroll
          for (int h = 0; h < 8; ++h) {
            const float4 w = *reinterpret_cast<const float4*>(s_gw + h * dim + 4 * c);
#pragma unroll
            for (int k = 0; k < ROWS; ++k)
              acc[k * 8 + h] += v[k][i].x * w.x + v[k][i].y * w.y + v[k][i].z * w.z + v[k][i].w * w.w;
          }
        }
      }
      const float tot = reduce16(acc, lane);
      const int idx = ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
      const int k = idx >> 3, h = idx & 7;
      if ((lane & 1) == 0 && r0 + k < rows) gout[(r0 + k) * 8 + h] = ub::sigmoidf_(tot + __ldg(gb + h));
    } else if (gates > 0) {
#pragma unroll
      for (int k = 0; k < ROWS; ++k) {
        for (int h = 0; h < gates; ++h) {
          float acc = 0.f;
#pragma unroll
          for (int i = 0; i < kMaxVec; ++i) {
            const int c = lane + 32 * i;
            if (c < nv) {
              const float4 w = *reinterpret_cast<const float4*>(s_gw + h * dim + 4 * c);
              acc += v[k][i].x * w.x + v[k][i].y * w.y + v[k][i].z * w.z + v[k][i].w * w.w;
            }
          }
          acc = ub::warp_sum(acc);
          if (lane == 0 && r0 + k < rows) gout[(r0 + k) * gates + h] = ub::sigmoidf_(acc + __ldg(gb + h));
        }
      }
    }
  }
}

// Band b covers columns [start[b], start[b+1]) of each row.
__global__ void __launch_bounds__(256) band_rms_norm_kernel(const float* __restrict__ x, long long rows, long long ldx,
                                                            const int* __restrict__ start, int bands,
                                                            const float* __restrict__ gamma, void* __restrict__ y,
                                                            long long ldy, int y_bf16,
                                                            const int* __restrict__ y_start) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  const long long total = rows * bands;
  for (long long wi = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5); wi < total; wi += warps) {
    const long long r = wi / bands;
    const int b = (int)(wi - r * bands);
    const int c0 = __ldg(start + b), c1 = __ldg(start + b + 1);
    const int o0 = y_start ? __ldg(y_start + b) : c0;
    const int n4 = (c1 - c0) >> 2;
    const float4* xr = reinterpret_cast<const float4*>(x + r * ldx + c0);
    float ss = 0.f;
    for (int i = lane; i < n4; i += 32) {
      const float4 v = __ldg(xr + i);
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    ss = ub::warp_sum(ss);
    const float inv = rsqrtf(ss / (float)(c1 - c0) + kEps);
    for (int i = lane; i < n4; i += 32) {
      const float4 v = __ldg(xr + i);
      const float4 g = __ldg(reinterpret_cast<const float4*>(gamma + c0) + i);
      store4(y, r * ldy + o0 + 4 * i, make_float4(v.x * inv * g.x, v.y * inv * g.y, v.z * inv * g.z, v.w * inv * g.w),
             y_bf16);
    }
  }
}

}  // namespace

extern "C" int unblend_rms_norm(const float* x, long long rows, int dim, const float* gamma, void* y, long long ldy,
                                int y_bf16, const float* gate_w, const float* gate_b, int gates, float* gate_out,
                                void* stream) {
  UB_REQUIRE(x && gamma && y && rows > 0 && dim > 0 && dim % 4 == 0 && dim <= 4 * 32 * kMaxVec);
  UB_REQUIRE(ldy >= dim && ldy % 4 == 0);
  UB_REQUIRE(gates >= 0 && gates <= kMaxGates && (gates == 0 || (gate_w && gate_b && gate_out)));
  UB_REQUIRE((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(gamma) & 15) == 0);
  UB_REQUIRE((reinterpret_cast<uintptr_t>(y) & (y_bf16 ? 7 : 15)) == 0);
  const size_t smem = (size_t)gates * dim * sizeof(float);
  UB_REQUIRE(smem <= 200 * 1024);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(rms_norm_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const long long blocks_needed = (rows + 15) / 16;
  const unsigned grid = (unsigned)(blocks_needed < 148LL * 8 ? blocks_needed : 148LL * 8);
  rms_norm_kernel<2><<<grid, 256, smem, ub::as_stream(stream)>>>(x, rows, dim, gamma, y, ldy, y_bf16 ? 1 : 0, gate_w,
                                                                 gate_b, gates, gate_out);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_band_rms_norm(const float* x, long long rows, long long ldx, const int* band_start, int bands,
                                     const float* gamma, void* y, long long ldy, int y_bf16, const int* y_start,
                                     void* stream) {
  UB_REQUIRE(x && band_start && gamma && y && rows > 0 && bands > 0 && ldx % 4 == 0 && ldy % 4 == 0);
  UB_REQUIRE((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(gamma) & 15) == 0);
  UB_REQUIRE((reinterpret_cast<uintptr_t>(y) & (y_bf16 ? 7 : 15)) == 0);
  const long long warps = rows * bands;
  const long long blocks_needed = (warps + 7) / 8;
  const unsigned grid = (unsigned)(blocks_needed < 148LL * 16 ? blocks_needed : 148LL * 16);
  band_rms_norm_kernel<<<grid, 256, 0, ub::as_stream(stream)>>>(x, rows, ldx, band_start, bands, gamma, y, ldy,
                                                               y_bf16 ? 1 : 0, y_start);
  UB_CHECK_LAUNCH();
  return 0;
}
