// Normalisation, statistics and elementwise kernels (HBM-streaming, fp32).
//
// GroupNorm(1, C) of the DConv branches (unblend/blocks.py:282-302), the
// transformer LayerNorms and sequence-global norm_out GroupNorm
// (unblend/transformer.py:225-236, 310-316), the HTDemucs input
// normalisation (unblend/htdemucs.py:669-678) and the DConv tail
// x + LayerScale * GLU(GN(z)) (unblend/blocks.py:293-317).
// Statistics accumulate in double so that fp32 parity holds for groups of
// millions of elements.
#include <cuda_bf16.h>

#include "common.cuh"

namespace {

__global__ void zero_f64_kernel(double* p, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    p[i] = 0.0;
}

// n floats from p, 16 bytes per store after a scalar head up to the first 16-byte boundary.
__global__ void zero_f32_kernel(float* p, long long n) {
  const long long head = (long long)((16 - ((uintptr_t)p & 15)) & 15) / 4;
  const long long h = head < n ? head : n;
  const long long t0 = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  const long long step = (long long)gridDim.x * blockDim.x;
  if (t0 < h) p[t0] = 0.f;
  float4* q = reinterpret_cast<float4*>(p + h);
  const long long n4 = (n - h) / 4;
  for (long long i = t0; i < n4; i += step) q[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (long long i = h + 4 * n4 + t0; i < n; i += step) p[i] = 0.f;
}

// count blocks of n floats at p + i * stride (small strided regions: padding rows).
__global__ void zero_f32_blocks_kernel(float* p, int count, long long stride, long long n) {
  const long long total = (long long)count * n;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x)
    p[(i / n) * stride + i % n] = 0.f;
}

// grid: (blocks_per_group, groups); one partial per block then a double atomic.
__global__ void group_sums_kernel(const float* __restrict__ x, double* stats, long long n) {
  const float* xg = x + (long long)blockIdx.y * n;
  double s1 = 0.0, s2 = 0.0;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    double v = (double)__ldg(xg + i);
    s1 += v;
    s2 += v * v;
  }
  s1 = ub::warp_sum_d(s1);
  s2 = ub::warp_sum_d(s2);
  __shared__ double sh[2][32];
  int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) {
    sh[0][wid] = s1;
    sh[1][wid] = s2;
  }
  __syncthreads();
  if (wid == 0) {
    int nw = blockDim.x >> 5;
    s1 = lane < nw ? sh[0][lane] : 0.0;
    s2 = lane < nw ? sh[1][lane] : 0.0;
    s1 = ub::warp_sum_d(s1);
    s2 = ub::warp_sum_d(s2);
    if (lane == 0) {
      atomicAdd(stats + 2 * blockIdx.y, s1);
      atomicAdd(stats + 2 * blockIdx.y + 1, s2);
    }
  }
}

__global__ void stats_finalize_kernel(const double* stats, float* out, int groups, double count,
                                      float eps, int unbiased, int std_mode) {
  int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= groups) return;
  double s = stats[2 * g], sq = stats[2 * g + 1];
  double mean = s / count;
  double var = (sq - s * mean) / (count - (unbiased ? 1.0 : 0.0));
  if (var < 0) var = 0;
  out[2 * g] = (float)mean;
  if (std_mode)
    out[2 * g + 1] = (float)sqrt(var);
  else
    out[2 * g + 1] = (float)(1.0 / sqrt(var + (double)eps));
}

__global__ void group_norm_apply_kernel(const float* __restrict__ x, float* __restrict__ y,
                                        const float* __restrict__ st, const float* __restrict__ gamma,
                                        const float* __restrict__ beta, long long rows, int c,
                                        long long rows_per_group, int act) {
  long long n = rows * c;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    long long r = i / c;
    int ch = (int)(i - r * c);
    long long g = r / rows_per_group;
    float v = (x[i] - st[2 * g]) * st[2 * g + 1];
    if (gamma) v = v * gamma[ch];
    if (beta) v = v + beta[ch];
    if (act == UNBLEND_ACT_GELU) v = ub::gelu_erf(v);
    if (act == UNBLEND_ACT_SWISH) v = v / (1.0f + expf(-v));
    y[i] = v;
  }
}

__global__ void dconv_tail_kernel(float* __restrict__ x, const float* __restrict__ z,
                                  const float* __restrict__ st, const float* __restrict__ gamma,
                                  const float* __restrict__ beta, const float* __restrict__ scale,
                                  long long groups, long long rows_per_group, int c, long long x_gs) {
  const long long n = groups * rows_per_group * c;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / c;
    const int ch = (int)(i - r * c);
    const long long g = r / rows_per_group;
    const long long rr = r - g * rows_per_group;
    const float mean = st[2 * g], rstd = st[2 * g + 1];
    const float2 zz = *reinterpret_cast<const float2*>(z + r * 2 * c + 2 * ch);
    const float va = (zz.x - mean) * rstd * gamma[2 * ch] + beta[2 * ch];
    const float vg = (zz.y - mean) * rstd * gamma[2 * ch + 1] + beta[2 * ch + 1];
    float* xp = x + g * x_gs + rr * c + ch;
    *xp = *xp + scale[ch] * (va * ub::sigmoid_approx(vg));
  }
}

// One warp per row; c <= 1024 and c % 32 == 0 not required.
// One warp per row. OutT float, or __nv_bfloat16 for a row that only feeds bf16 GEMMs.
template <typename OutT>
__global__ void layer_norm_kernel(const float* __restrict__ x, OutT* __restrict__ y,
                                  const float* __restrict__ gamma, const float* __restrict__ beta,
                                  const float* __restrict__ pos, float pos_scale, long long pos_rows,
                                  long long rows, int c) {
  long long row = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5);
  int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* xr = x + row * c;
  // Fixed trip count with a predicate so that vals[] stays in registers
  // (a runtime-bounded loop indexes it dynamically, i.e. in local memory).
  float vals[32];
  const int nper = (c + 31) / 32;
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int ch = lane + 32 * j;
    const float v = (j < nper && ch < c) ? xr[ch] : 0.f;
    vals[j] = v;
    s += v;
  }
  const float mean = ub::warp_sum(s) / c;
  float s2 = 0.f;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int ch = lane + 32 * j;
    const float d = (j < nper && ch < c) ? vals[j] - mean : 0.f;
    s2 += d * d;
  }
  const float var = ub::warp_sum(s2) / c;
  const float rstd = rsqrtf(var + 1e-5f);
  OutT* yr = y + row * c;
  const float* pr = pos ? pos + (row % pos_rows) * c : nullptr;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int ch = lane + 32 * j;
    if (j < nper && ch < c) {
      float v = (vals[j] - mean) * rstd * gamma[ch] + beta[ch];
      if (pr) v += pos_scale * pr[ch];
      if constexpr (sizeof(OutT) == 2)
        yr[ch] = __float2bfloat16_rn(v);
      else
        yr[ch] = v;
    }
  }
}

__global__ void add_kernel(const float* __restrict__ a, const float* __restrict__ b, float* y,
                           long long n, long long period, float alpha) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    y[i] = a[i] + alpha * b[i % period];
}

__global__ void time_input_kernel(const float* __restrict__ mix, float* __restrict__ xt,
                                  const float* __restrict__ st, int batch, int length, int length_pad) {
  long long n = (long long)batch * length_pad;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    int b = (int)(i / length_pad);
    int t = (int)(i - (long long)b * length_pad);
    float2 o = make_float2(0.f, 0.f);
    if (t < length) {
      float mean = st[2 * b], den = 1e-5f + st[2 * b + 1];
      const float* mb = mix + (long long)b * 2 * length;
      o.x = (mb[t] - mean) / den;
      o.y = (mb[length + t] - mean) / den;
    }
    *reinterpret_cast<float2*>(xt + 2 * i) = o;
  }
}

// y[i] = bf16(x[i]) (round to nearest even), four elements per thread.
__global__ void cast_bf16_kernel(const float4* __restrict__ x, uint2* __restrict__ y, long long n4) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
       i += (long long)gridDim.x * blockDim.x) {
    const float4 v = __ldg(x + i);
    __nv_bfloat162 p0 = __floats2bfloat162_rn(v.x, v.y);
    __nv_bfloat162 p1 = __floats2bfloat162_rn(v.z, v.w);
    uint2 o;
    o.x = *reinterpret_cast<uint32_t*>(&p0);
    o.y = *reinterpret_cast<uint32_t*>(&p1);
    y[i] = o;
  }
}

// Four channels per thread with 32-bit index arithmetic (the launchers use
// these when c is a multiple of 4 and the element count fits in 31 bits; the
// per-element 64-bit divisions of the scalar kernels dominated their time).
__global__ void group_norm_apply4_kernel(const float4* __restrict__ x, float4* __restrict__ y,
                                         const float* __restrict__ st, const float* __restrict__ gamma,
                                         const float* __restrict__ beta, int n4, int c4, int rows_per_group,
                                         int act) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x) {
    const int r = i / c4, q = i - r * c4;
    const int g = r / rows_per_group;
    const float m = __ldg(st + 2 * g), rs = __ldg(st + 2 * g + 1);
    const float4 v = x[i];
    float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float t = (e[k] - m) * rs;
      if (gamma) t = t * __ldg(gamma + 4 * q + k);
      if (beta) t = t + __ldg(beta + 4 * q + k);
      if (act == UNBLEND_ACT_GELU) t = ub::gelu_erf(t);
      if (act == UNBLEND_ACT_SWISH) t = t / (1.0f + expf(-t));
      e[k] = t;
    }
    y[i] = make_float4(e[0], e[1], e[2], e[3]);
  }
}

__global__ void dconv_tail4_kernel(float* __restrict__ x, const float4* __restrict__ z,
                                   const float* __restrict__ st, const float4* __restrict__ gamma,
                                   const float4* __restrict__ beta, const float4* __restrict__ scale, int n4,
                                   int c4, int rows_per_group, long long x_gs) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x) {
    const int r = i / c4, q = i - r * c4;
    const int g = r / rows_per_group, rr = r - g * rows_per_group;
    const float mean = __ldg(st + 2 * g), rstd = __ldg(st + 2 * g + 1);
    // z row r: 2c values, (value, gate) interleaved per channel.
    const float4 z0 = __ldg(z + 2LL * i), z1 = __ldg(z + 2LL * i + 1);
    const float4 g0 = __ldg(gamma + 2 * q), g1 = __ldg(gamma + 2 * q + 1);
    const float4 b0 = __ldg(beta + 2 * q), b1 = __ldg(beta + 2 * q + 1);
    const float4 sc = __ldg(scale + q);
    const float zv[8] = {z0.x, z0.y, z0.z, z0.w, z1.x, z1.y, z1.z, z1.w};
    const float gv[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
    const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    const float sv[4] = {sc.x, sc.y, sc.z, sc.w};
    float4* xp = reinterpret_cast<float4*>(x + (long long)g * x_gs + (long long)rr * (4 * c4)) + q;
    const float4 xv = *xp;
    float o[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float va = (zv[2 * k] - mean) * rstd * gv[2 * k] + bv[2 * k];
      const float vg = (zv[2 * k + 1] - mean) * rstd * gv[2 * k + 1] + bv[2 * k + 1];
      o[k] = o[k] + sv[k] * (va * ub::sigmoid_approx(vg));
    }
    *xp = make_float4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace

extern "C" int unblend_zero_f64(double* p, long long n, void* stream) {
  UB_REQUIRE(p && n >= 0);
  if (n == 0) return 0;
  zero_f64_kernel<<<ub::grid_1d(n, 256), 256, 0, ub::as_stream(stream)>>>(p, n);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_zero_f32(float* p, long long n, int count, long long stride, void* stream) {
  UB_REQUIRE(p && n >= 0 && count >= 1 && ((uintptr_t)p & 3) == 0 && (count == 1 || stride >= n));
  if (n == 0) return 0;
  if (count == 1)
    zero_f32_kernel<<<ub::grid_1d(n / 4 + 1, 256), 256, 0, ub::as_stream(stream)>>>(p, n);
  else
    zero_f32_blocks_kernel<<<ub::grid_1d((long long)count * n, 256), 256, 0, ub::as_stream(stream)>>>(
        p, count, stride, n);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_group_sums(const float* x, double* stats, int groups, long long n, void* stream) {
  UB_REQUIRE(x && stats && groups > 0 && n > 0 && groups < 65536);
  long long per = (n + 255) / 256;
  int bx = (int)(per < 256 ? per : 256);
  dim3 grid(bx, groups);
  group_sums_kernel<<<grid, 256, 0, ub::as_stream(stream)>>>(x, stats, n);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_stats_finalize(const double* stats, float* out, int groups, double count,
                                      float eps, int unbiased, int std_mode, void* stream) {
  UB_REQUIRE(stats && out && groups > 0 && count > (unbiased ? 1.0 : 0.0));
  stats_finalize_kernel<<<(groups + 127) / 128, 128, 0, ub::as_stream(stream)>>>(
      stats, out, groups, count, eps, unbiased, std_mode);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_group_norm_apply(const float* x, float* y, const float* stats2, const float* gamma,
                                        const float* beta, long long rows, int c, long long rows_per_group,
                                        int act, void* stream) {
  UB_REQUIRE(x && y && stats2 && rows > 0 && c > 0 && rows_per_group > 0);
  UB_REQUIRE(act == UNBLEND_ACT_NONE || act == UNBLEND_ACT_GELU || act == UNBLEND_ACT_SWISH);
  if (c % 4 == 0 && rows * c < (1LL << 31) && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(y) & 15) == 0) {
    const int n4 = (int)(rows * c / 4);
    group_norm_apply4_kernel<<<ub::grid_1d(n4, 256), 256, 0, ub::as_stream(stream)>>>(
        reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(y), stats2, gamma, beta, n4, c / 4,
        (int)rows_per_group, act);
    UB_CHECK_LAUNCH();
    return 0;
  }
  group_norm_apply_kernel<<<ub::grid_1d(rows * c, 256), 256, 0, ub::as_stream(stream)>>>(
      x, y, stats2, gamma, beta, rows, c, rows_per_group, act);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_dconv_tail(float* x, const float* z, const float* stats2, const float* gamma,
                                  const float* beta, const float* scale, long long groups,
                                  long long rows_per_group, int c, long long x_group_stride, void* stream) {
  UB_REQUIRE(x && z && stats2 && gamma && beta && scale && groups > 0 && rows_per_group > 0 && c > 0);
  UB_REQUIRE(x_group_stride >= rows_per_group * c);
  const long long n = groups * rows_per_group * c;
  if (c % 4 == 0 && n < (1LL << 31) && x_group_stride % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(z) & 15) == 0 && (reinterpret_cast<uintptr_t>(gamma) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(beta) & 15) == 0 && (reinterpret_cast<uintptr_t>(scale) & 15) == 0) {
    const int n4 = (int)(n / 4);
    dconv_tail4_kernel<<<ub::grid_1d(n4, 256), 256, 0, ub::as_stream(stream)>>>(
        x, reinterpret_cast<const float4*>(z), stats2, reinterpret_cast<const float4*>(gamma),
        reinterpret_cast<const float4*>(beta), reinterpret_cast<const float4*>(scale), n4, c / 4,
        (int)rows_per_group, x_group_stride);
    UB_CHECK_LAUNCH();
    return 0;
  }
  dconv_tail_kernel<<<ub::grid_1d(groups * rows_per_group * c, 256), 256, 0, ub::as_stream(stream)>>>(
      x, z, stats2, gamma, beta, scale, groups, rows_per_group, c, x_group_stride);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_layer_norm(const float* x, float* y, const float* gamma, const float* beta,
                                  const float* pos, float pos_scale, long long pos_rows, long long rows,
                                  int c, void* stream) {
  UB_REQUIRE(x && y && gamma && beta && rows > 0 && c > 0 && c <= 1024);
  UB_REQUIRE(!pos || pos_rows > 0);
  unsigned grid = (unsigned)((rows + 7) / 8);
  layer_norm_kernel<float><<<grid, 256, 0, ub::as_stream(stream)>>>(x, y, gamma, beta, pos, pos_scale,
                                                                      pos_rows, rows, c);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_layer_norm_bf16(const float* x, void* y, const float* gamma, const float* beta,
                                       const float* pos, float pos_scale, long long pos_rows, long long rows,
                                       int c, void* stream) {
  UB_REQUIRE(x && y && gamma && beta && rows > 0 && c > 0 && c <= 1024);
  UB_REQUIRE(!pos || pos_rows > 0);
  unsigned grid = (unsigned)((rows + 7) / 8);
  layer_norm_kernel<__nv_bfloat16><<<grid, 256, 0, ub::as_stream(stream)>>>(
      x, reinterpret_cast<__nv_bfloat16*>(y), gamma, beta, pos, pos_scale, pos_rows, rows, c);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_add(const float* a, const float* b, float* y, long long n, long long b_period,
                           float alpha, void* stream) {
  UB_REQUIRE(a && b && y && n > 0 && b_period > 0);
  add_kernel<<<ub::grid_1d(n, 256), 256, 0, ub::as_stream(stream)>>>(a, b, y, n, b_period, alpha);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_cast_bf16(const float* x, void* y, long long n, void* stream) {
  UB_REQUIRE(x && y && n > 0 && n % 4 == 0);
  UB_REQUIRE((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(y) & 7) == 0);
  cast_bf16_kernel<<<ub::grid_1d(n / 4, 256), 256, 0, ub::as_stream(stream)>>>(
      reinterpret_cast<const float4*>(x), reinterpret_cast<uint2*>(y), n / 4);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_time_input(const float* mix, float* xt, const float* stats2, int batch, int length,
                                  int length_pad, void* stream) {
  UB_REQUIRE(mix && xt && stats2 && batch > 0 && length > 0 && length_pad >= length);
  time_input_kernel<<<ub::grid_1d((long long)batch * length_pad, 256), 256, 0, ub::as_stream(stream)>>>(
      mix, xt, stats2, batch, length, length_pad);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_mean_std(const float* x, double* work, float* out, int batch, long long n,
                                void* stream) {
  int rc = unblend_zero_f64(work, 2LL * batch, stream);
  if (rc) return rc;
  rc = unblend_group_sums(x, work, batch, n, stream);
  if (rc) return rc;
  return unblend_stats_finalize(work, out, batch, (double)n, 0.f, 1, 1, stream);
}

namespace {
__global__ void standardize_kernel(const float* __restrict__ x, float* __restrict__ y,
                                   const float* __restrict__ st, long long n_per_batch, int batch) {
  long long n = n_per_batch * batch;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    long long b = i / n_per_batch;
    y[i] = (x[i] - st[2 * b]) / (1e-5f + st[2 * b + 1]);
  }
}
}  // namespace

extern "C" int unblend_standardize(const float* x, float* y, const float* stats2, long long n_per_batch,
                                   int batch, void* stream) {
  UB_REQUIRE(x && y && stats2 && n_per_batch > 0 && batch > 0);
  standardize_kernel<<<ub::grid_1d(n_per_batch * batch, 256), 256, 0, ub::as_stream(stream)>>>(
      x, y, stats2, n_per_batch, batch);
  UB_CHECK_LAUNCH();
  return 0;
}

// ---------------------------------------------------------------------------
// Allocation-free variant of unblend_mean_std.
//
// unblend_mean_std needs a double[2 * batch] accumulator from its caller. Some
// callers cannot provide one: code running on a real-time audio thread, where
// cudaMalloc can block on a device-wide synchronisation for an unbounded time,
// and hosts that embed this library under a memory manager that owns every
// device allocation. For them the accumulator lives in this file-scope device
// array instead: UNBLEND_NOALLOC_MAX_BATCH batch items at most (64 KiB), held
// by every GPU that loads the library until the process exits.
static __device__ __align__(256) double g_mean_std_scratch[2 * UNBLEND_NOALLOC_MAX_BATCH];

#include <cuda.h>

#include <mutex>

namespace {
std::mutex g_scratch_mutex;

// The array's device address is cached per device together with the CUDA
// context it was resolved in. A host that resets the device
// (cudaDeviceReset) or drives it through a context of its own gets a new
// context, where the array can sit at another address: the address is looked
// up again whenever the current context differs from the cached one.
struct ScratchSlot {
  CUcontext ctx;
  double* addr;
};
ScratchSlot g_scratch[64] = {};

using CtxGetCurrent = CUresult (*)(CUcontext*);

// cuCtxGetCurrent through the runtime's driver entry-point query (no link
// dependency on the driver library); null if the driver does not provide it.
CtxGetCurrent ctx_get_current() {
  static CtxGetCurrent fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<CtxGetCurrent>(p);
  }();
  return fn;
}

// Device address of the scratch array in the current context. In host code the
// array's name is only a host-side stand-in, so the address is resolved with
// the device current: on the first call per device, and again after the
// device's context changed.
int scratch_for_current_device(double** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= 64) return UNBLEND_ERR_INVALID;
  CtxGetCurrent get = ctx_get_current();
  CUcontext ctx = nullptr;
  if (get && get(&ctx) != CUDA_SUCCESS) ctx = nullptr;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  ScratchSlot& slot = g_scratch[dev];
  if (!slot.addr || !ctx || slot.ctx != ctx) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_mean_std_scratch);
    if (e != cudaSuccess) return (int)e;
    // The lookup makes the device's primary context current if none was.
    if (get && get(&ctx) != CUDA_SUCCESS) ctx = nullptr;
    slot.ctx = ctx;
    slot.addr = static_cast<double*>(p);
  }
  *out = slot.addr;
  return 0;
}
}  // namespace

extern "C" int unblend_mean_std_noalloc(const float* x, float* out, int batch, long long n, void* stream) {
  UB_REQUIRE(x && out && batch > 0 && n > 1);
  if (batch > UNBLEND_NOALLOC_MAX_BATCH) return UNBLEND_ERR_TOO_LARGE;
  double* scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
  if (rc) return rc;
  // The array keeps the previous call's sums: clear the part this call uses.
  rc = unblend_zero_f64(scratch, 2LL * batch, stream);
  if (rc) return rc;
  rc = unblend_group_sums(x, scratch, batch, n, stream);
  if (rc) return rc;
  return unblend_stats_finalize(scratch, out, batch, (double)n, 0.f, 1, 1, stream);
}
