// Fused DConv residual branch (unblend/blocks.py:238-317), fp32, HBM-streaming.
//
// One DConv layer is  x += LayerScale * GLU(GN2(W2 * GELU(GN1(conv_k3_dil(x)))))
// with GroupNorm(1) statistics per group (a (batch, frequency) row of the
// frequency branch, or a batch item of the time branch). The hidden width is
// C/8, so both contractions are far too thin for tensor cores to pay; the
// cost is moving x. Three kernels:
//   dconv_conv1   h = conv_k3_dil(x) with GN1 sums (x tile + weights in smem)
//   dconv_z_stats GN2 sums of z = W2 * GELU(GN1(h)) + b2, z never stored
//   dconv_apply   recompute z, x += scale * GLU(GN2(z)) in place
// x element (g, r, c) is at x + g * x_gs + r * C + c; h is contiguous
// [groups, rows, H]. W1 is [H, 3, C]; W2 is [2C, H] with rows interleaved as
// (value 0, gate 0, value 1, gate 1, ...), GN2 affine in the same order.
#include "common.cuh"

namespace {

constexpr int ROWS = 128;  // rows per CTA, one thread per row

template <int MAXH>
__global__ void __launch_bounds__(ROWS) dconv_conv1_kernel(const float* __restrict__ x, long long x_gs, int rows,
                                                           int C, const float* __restrict__ w1,
                                                           const float* __restrict__ b1, int H, int dil,
                                                           float* __restrict__ h, double* __restrict__ stats) {
  extern __shared__ __align__(16) float sm[];
  const int CP = C + 4;  // padded row stride (keeps 16-byte alignment)
  float* xs = sm;                                  // [ROWS + 2*dil][CP]
  float* ws = sm + (ROWS + 2 * dil) * CP;          // [H][3][C]
  const int g = blockIdx.y;
  const int r0 = blockIdx.x * ROWS;
  const float* xg = x + (long long)g * x_gs;
  const int nrows = ROWS + 2 * dil;
  // Stage the x rows [r0 - dil, r0 + ROWS + dil) (zero outside [0, rows)).
  const int c4 = C / 4;
  for (int i = threadIdx.x; i < nrows * c4; i += ROWS) {
    const int rr = i / c4, cc = (i - rr * c4) * 4;
    const int r = r0 - dil + rr;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r >= 0 && r < rows) v = *reinterpret_cast<const float4*>(xg + (long long)r * C + cc);
    *reinterpret_cast<float4*>(xs + rr * CP + cc) = v;
  }
  for (int i = threadIdx.x; i < H * 3 * C; i += ROWS) ws[i] = w1[i];
  __syncthreads();
  const int lr = threadIdx.x;
  const int r = r0 + lr;
  float acc[MAXH];
#pragma unroll
  for (int j = 0; j < MAXH; ++j) acc[j] = (j < H) ? __ldg(b1 + j) : 0.f;
  for (int t = 0; t < 3; ++t) {
    const float* xr = xs + (lr + t * dil) * CP;
    for (int c = 0; c < C; c += 4) {
      const float4 xv = *reinterpret_cast<const float4*>(xr + c);
#pragma unroll
      for (int j = 0; j < MAXH; ++j) {
        if (j < H) {
          const float4 wv = *reinterpret_cast<const float4*>(ws + (j * 3 + t) * C + c);
          acc[j] = fmaf(xv.x, wv.x, fmaf(xv.y, wv.y, fmaf(xv.z, wv.z, fmaf(xv.w, wv.w, acc[j]))));
        }
      }
    }
  }
  float s1 = 0.f, s2 = 0.f;
  if (r < rows) {
    float* hr = h + ((long long)g * rows + r) * H;
#pragma unroll
    for (int j = 0; j < MAXH; ++j) {
      if (j < H) {
        hr[j] = acc[j];
        s1 += acc[j];
        s2 += acc[j] * acc[j];
      }
    }
  }
  s1 = ub::warp_sum(s1);
  s2 = ub::warp_sum(s2);
  __shared__ float red[2][ROWS / 32];
  if ((threadIdx.x & 31) == 0) {
    red[0][threadIdx.x >> 5] = s1;
    red[1][threadIdx.x >> 5] = s2;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double a = 0, b = 0;
    for (int i = 0; i < ROWS / 32; ++i) {
      a += red[0][i];
      b += red[1][i];
    }
    atomicAdd(stats + 2 * g, a);
    atomicAdd(stats + 2 * g + 1, b);
  }
}

// GELU(GN1(h)) of one row into registers.
template <int MAXH>
__device__ __forceinline__ void load_act(const float* __restrict__ hr, int H, float mean, float rstd,
                                         const float* __restrict__ g1w, const float* __restrict__ g1b,
                                         float (&a)[MAXH]) {
#pragma unroll
  for (int j = 0; j < MAXH; ++j) {
    float v = 0.f;
    if (j < H) v = ub::gelu_erf((hr[j] - mean) * rstd * __ldg(g1w + j) + __ldg(g1b + j));
    a[j] = v;
  }
}

template <int MAXH>
__device__ __forceinline__ float dot_row(const float* __restrict__ wrow, const float (&a)[MAXH], int H, float b) {
  float z = b;
#pragma unroll
  for (int j = 0; j < MAXH; ++j)
    if (j < H) z = fmaf(wrow[j], a[j], z);
  return z;
}

template <int MAXH>
__global__ void __launch_bounds__(ROWS) dconv_z_stats_kernel(const float* __restrict__ h, int rows, int H, int C,
                                                             const float* __restrict__ st1,
                                                             const float* __restrict__ g1w,
                                                             const float* __restrict__ g1b,
                                                             const float* __restrict__ w2,
                                                             const float* __restrict__ b2,
                                                             double* __restrict__ stats2) {
  extern __shared__ __align__(16) float sm[];
  float* ws = sm;  // [2C][H]
  float* bs = sm + 2 * C * H;
  for (int i = threadIdx.x; i < 2 * C * H; i += ROWS) ws[i] = w2[i];
  for (int i = threadIdx.x; i < 2 * C; i += ROWS) bs[i] = b2[i];
  __syncthreads();
  const int g = blockIdx.y;
  const int r = blockIdx.x * ROWS + threadIdx.x;
  float s1 = 0.f, s2 = 0.f;
  if (r < rows) {
    float a[MAXH];
    load_act<MAXH>(h + ((long long)g * rows + r) * H, H, st1[2 * g], st1[2 * g + 1], g1w, g1b, a);
    for (int n = 0; n < 2 * C; ++n) {
      const float z = dot_row<MAXH>(ws + n * H, a, H, bs[n]);
      s1 += z;
      s2 += z * z;
    }
  }
  s1 = ub::warp_sum(s1);
  s2 = ub::warp_sum(s2);
  __shared__ float red[2][ROWS / 32];
  if ((threadIdx.x & 31) == 0) {
    red[0][threadIdx.x >> 5] = s1;
    red[1][threadIdx.x >> 5] = s2;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double a0 = 0, a1 = 0;
    for (int i = 0; i < ROWS / 32; ++i) {
      a0 += red[0][i];
      a1 += red[1][i];
    }
    atomicAdd(stats2 + 2 * g, a0);
    atomicAdd(stats2 + 2 * g + 1, a1);
  }
}

template <int MAXH>
__global__ void __launch_bounds__(ROWS) dconv_apply_kernel(float* __restrict__ x, long long x_gs,
                                                           const float* __restrict__ h, int rows, int H, int C,
                                                           const float* __restrict__ st1,
                                                           const float* __restrict__ g1w,
                                                           const float* __restrict__ g1b,
                                                           const float* __restrict__ w2,
                                                           const float* __restrict__ b2,
                                                           const float* __restrict__ st2,
                                                           const float* __restrict__ g2w,
                                                           const float* __restrict__ g2b,
                                                           const float* __restrict__ scale) {
  extern __shared__ __align__(16) float sm[];
  float* ws = sm;             // [2C][H]
  float* bs = ws + 2 * C * H; // [2C]
  float* gw = bs + 2 * C;     // [2C] GN2 gamma * rstd
  float* gb = gw + 2 * C;     // [2C] GN2 beta - mean * rstd * gamma
  float* sc = gb + 2 * C;     // [C]
  const int g = blockIdx.y;
  const float mean2 = st2[2 * g], rstd2 = st2[2 * g + 1];
  for (int i = threadIdx.x; i < 2 * C * H; i += ROWS) ws[i] = w2[i];
  for (int i = threadIdx.x; i < 2 * C; i += ROWS) {
    bs[i] = b2[i];
    gw[i] = g2w[i];
    gb[i] = g2b[i];
  }
  for (int i = threadIdx.x; i < C; i += ROWS) sc[i] = scale[i];
  __syncthreads();
  const int r = blockIdx.x * ROWS + threadIdx.x;
  if (r >= rows) return;
  float a[MAXH];
  load_act<MAXH>(h + ((long long)g * rows + r) * H, H, st1[2 * g], st1[2 * g + 1], g1w, g1b, a);
  float* xr = x + (long long)g * x_gs + (long long)r * C;
  for (int c = 0; c < C; c += 4) {
    float4 xv = *reinterpret_cast<float4*>(xr + c);
    float o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int n = 2 * (c + e);
      const float zv = dot_row<MAXH>(ws + n * H, a, H, bs[n]);
      const float zg = dot_row<MAXH>(ws + (n + 1) * H, a, H, bs[n + 1]);
      const float v = (zv - mean2) * rstd2 * gw[n] + gb[n];
      const float gt = (zg - mean2) * rstd2 * gw[n + 1] + gb[n + 1];
      o[e] = sc[c + e] * (v * ub::sigmoidf_(gt));
    }
    xv.x += o[0];
    xv.y += o[1];
    xv.z += o[2];
    xv.w += o[3];
    *reinterpret_cast<float4*>(xr + c) = xv;
  }
}

int maxh_for(int H) { return H <= 8 ? 8 : H <= 16 ? 16 : H <= 32 ? 32 : H <= 64 ? 64 : 0; }

}  // namespace

extern "C" int unblend_dconv_conv1(const float* x, long long x_gs, int groups, int rows, int c, const float* w1,
                                   const float* b1, int hid, int dil, float* h, double* stats, void* stream) {
  UB_REQUIRE(x && w1 && b1 && h && stats && groups > 0 && rows > 0 && c > 0 && c % 4 == 0);
  UB_REQUIRE(hid > 0 && dil > 0 && dil <= 8 && groups < 65536 && x_gs >= (long long)rows * c);
  const int mh = maxh_for(hid);
  UB_REQUIRE(mh > 0);
  const size_t smem = sizeof(float) * ((size_t)(ROWS + 2 * dil) * (c + 4) + (size_t)hid * 3 * c);
  UB_REQUIRE(smem <= 220 * 1024);
  dim3 grid((rows + ROWS - 1) / ROWS, groups);
  cudaStream_t st = ub::as_stream(stream);
#define UB_LAUNCH(MH)                                                                                         \
  {                                                                                                           \
    cudaFuncSetAttribute(dconv_conv1_kernel<MH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);    \
    dconv_conv1_kernel<MH><<<grid, ROWS, smem, st>>>(x, x_gs, rows, c, w1, b1, hid, dil, h, stats);           \
  }
  if (mh == 8) UB_LAUNCH(8) else if (mh == 16) UB_LAUNCH(16) else if (mh == 32) UB_LAUNCH(32) else UB_LAUNCH(64)
#undef UB_LAUNCH
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_dconv_z_stats(const float* h, int groups, int rows, int hid, int c, const float* st1,
                                     const float* g1w, const float* g1b, const float* w2, const float* b2,
                                     double* stats2, void* stream) {
  UB_REQUIRE(h && st1 && g1w && g1b && w2 && b2 && stats2 && groups > 0 && rows > 0 && c > 0 && hid > 0);
  UB_REQUIRE(groups < 65536);
  const int mh = maxh_for(hid);
  UB_REQUIRE(mh > 0);
  const size_t smem = sizeof(float) * ((size_t)2 * c * hid + 2 * c);
  UB_REQUIRE(smem <= 220 * 1024);
  dim3 grid((rows + ROWS - 1) / ROWS, groups);
  cudaStream_t st = ub::as_stream(stream);
#define UB_LAUNCH(MH)                                                                                           \
  {                                                                                                             \
    cudaFuncSetAttribute(dconv_z_stats_kernel<MH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);    \
    dconv_z_stats_kernel<MH><<<grid, ROWS, smem, st>>>(h, rows, hid, c, st1, g1w, g1b, w2, b2, stats2);         \
  }
  if (mh == 8) UB_LAUNCH(8) else if (mh == 16) UB_LAUNCH(16) else if (mh == 32) UB_LAUNCH(32) else UB_LAUNCH(64)
#undef UB_LAUNCH
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_dconv_apply(float* x, long long x_gs, const float* h, int groups, int rows, int hid, int c,
                                   const float* st1, const float* g1w, const float* g1b, const float* w2,
                                   const float* b2, const float* st2, const float* g2w, const float* g2b,
                                   const float* scale, void* stream) {
  UB_REQUIRE(x && h && st1 && g1w && g1b && w2 && b2 && st2 && g2w && g2b && scale);
  UB_REQUIRE(groups > 0 && rows > 0 && c > 0 && c % 4 == 0 && hid > 0 && groups < 65536);
  UB_REQUIRE(x_gs >= (long long)rows * c && x_gs % 4 == 0);
  const int mh = maxh_for(hid);
  UB_REQUIRE(mh > 0);
  const size_t smem = sizeof(float) * ((size_t)2 * c * hid + 6 * (size_t)c + c);
  UB_REQUIRE(smem <= 220 * 1024);
  dim3 grid((rows + ROWS - 1) / ROWS, groups);
  cudaStream_t st = ub::as_stream(stream);
#define UB_LAUNCH(MH)                                                                                         \
  {                                                                                                           \
    cudaFuncSetAttribute(dconv_apply_kernel<MH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);    \
    dconv_apply_kernel<MH><<<grid, ROWS, smem, st>>>(x, x_gs, h, rows, hid, c, st1, g1w, g1b, w2, b2, st2,    \
                                                     g2w, g2b, scale);                                        \
  }
  if (mh == 8) UB_LAUNCH(8) else if (mh == 16) UB_LAUNCH(16) else if (mh == 32) UB_LAUNCH(32) else UB_LAUNCH(64)
#undef UB_LAUNCH
  UB_CHECK_LAUNCH();
  return 0;
}
