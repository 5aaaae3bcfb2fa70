// Generic implicit-GEMM convolution, fp32 SIMT (CUDA cores).
//
// Every Conv1d / Conv2d / ConvTranspose phase / Linear of the HTDemucs forward
// (unblend/blocks.py:461-467, 688-695, 297-300; unblend/transformer.py:290-301)
// can run here: output positions are the GEMM M dimension, output channels N,
// and (kh, kw, c_in) the K dimension gathered on the fly from a channels-last
// input with zero padding. Fused prologue (GroupNorm+GELU or a skip add on the
// loaded input) and epilogue (bias, GELU/GLU, LayerScale residual, GroupNorm
// statistics). This is the exact-fp32 path; dense layers also have a
// tensor-core path (tcgen05) built on the same parameter block.
#include "common.cuh"

namespace {

constexpr int BM = 128;
constexpr int BN = 64;
constexpr int BK = 16;
constexpr int NT = 256;

struct ConvArgs {
  UnblendConvParams p;
  const float* x;
  const float* w;
  const float* bias;
  float* y;
  long long M;
  int K;
};

__device__ __forceinline__ float load_a(const ConvArgs& a, int b, int hi, int wi, int ci) {
  const UnblendConvParams& p = a.p;
  long long off = (long long)b * p.in_sb + (long long)hi * p.in_sh + (long long)wi * p.in_sw + ci;
  float v = __ldg(a.x + off);
  if (p.prologue == UNBLEND_PRO_GN_GELU) {
    int g = p.pro_group_per_h ? b * p.h_in + hi : b;
    v = (v - __ldg(p.pro_stats + 2 * g)) * __ldg(p.pro_stats + 2 * g + 1);
    v = ub::gelu_erf(v * __ldg(p.pro_gamma + ci) + __ldg(p.pro_beta + ci));
  } else if (p.prologue == UNBLEND_PRO_ADD) {
    v += __ldg(p.pro_x2 + off);
  }
  return v;
}

__global__ void __launch_bounds__(NT) conv_simt_kernel(ConvArgs a) {
  const UnblendConvParams& p = a.p;
  __shared__ __align__(16) float As[2][BK][BM + 4];
  __shared__ __align__(16) float Bs[2][BK][BN + 4];

  const int tid = threadIdx.x;
  const long long m0 = (long long)blockIdx.x * BM;
  const int n0 = blockIdx.y * BN;

  // A-load role: one output position, 8 consecutive k.
  const int am = tid >> 1;
  const int ak = (tid & 1) * 8;
  const long long m = m0 + am;
  const bool mvalid = m < a.M;
  int wo = 0, ho = 0, b = 0;
  if (mvalid) {
    wo = (int)(m % p.w_out);
    long long t = m / p.w_out;
    ho = (int)(t % p.h_out);
    b = (int)(t / p.h_out);
  }
  const int hbase = ho * p.sh - p.ph;
  const int wbase = wo * p.sw - p.pw;

  // B-load role: one output channel, 4 consecutive k.
  const int bn = tid >> 2;
  const int bk = (tid & 3) * 4;
  const int nrow = n0 + bn;
  const float* wrow = a.w + (long long)nrow * a.K;

  float ra[8], rb[4];
  auto load_tiles = [&](int k0) {
    int k = k0 + ak;
    int tap = k / p.c_in;
    int ci = k - tap * p.c_in;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float v = 0.f;
      if (mvalid && k + i < a.K) {
        int kh = tap / p.kw;
        int kwi = tap - kh * p.kw;
        int hi = hbase + kh * p.dh;
        int wi = wbase + kwi * p.dw;
        if (hi >= 0 && hi < p.h_in && wi >= 0 && wi < p.w_in) v = load_a(a, b, hi, wi, ci);
      }
      ra[i] = v;
      if (++ci == p.c_in) { ci = 0; ++tap; }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int kk = k0 + bk + j;
      rb[j] = (nrow < p.n_out && kk < a.K) ? __ldg(wrow + kk) : 0.f;
    }
  };
  auto store_tiles = [&](int buf) {
#pragma unroll
    for (int i = 0; i < 8; ++i) As[buf][ak + i][am] = ra[i];
#pragma unroll
    for (int j = 0; j < 4; ++j) Bs[buf][bk + j][bn] = rb[j];
  };

  const int tx = tid & 15;  // N direction: 4 columns each
  const int ty = tid >> 4;  // M direction: 8 rows each
  float acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  const int ktiles = (a.K + BK - 1) / BK;
  load_tiles(0);
  store_tiles(0);
  __syncthreads();
  for (int kt = 0; kt < ktiles; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < ktiles) load_tiles((kt + 1) * BK);
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 8]);
      float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 8 + 4]);
      float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
      float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      float bv[4] = {b0.x, b0.y, b0.z, b0.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (kt + 1 < ktiles) store_tiles(buf ^ 1);
    __syncthreads();
  }

  // Epilogue.
  const bool glu = p.act == UNBLEND_ACT_GLU;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const long long mm = m0 + ty * 8 + i;
    const bool rv = mm < a.M;
    int owo = 0, oho = 0, ob = 0;
    if (rv) {
      owo = (int)(mm % p.w_out);
      long long t = mm / p.w_out;
      oho = (int)(t % p.h_out);
      ob = (int)(t / p.h_out);
    }
    const long long rowoff = (long long)ob * p.out_sb + (long long)oho * p.out_sh + (long long)owo * p.out_sw;
    float s1 = 0.f, s2 = 0.f;
    float vals[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int n = n0 + tx * 4 + j;
      float v = acc[i][j];
      if (n < p.n_out && a.bias) v += __ldg(a.bias + n);
      if (p.act == UNBLEND_ACT_GELU) v = ub::gelu_erf(v);
      vals[j] = v;
    }
    const int nouts = glu ? 2 : 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (j >= nouts) break;
      int n = glu ? (n0 + tx * 4) / 2 + j : n0 + tx * 4 + j;
      int ncount = glu ? p.n_out / 2 : p.n_out;
      float v = glu ? vals[2 * j] * ub::sigmoid_approx(vals[2 * j + 1]) : vals[j];
      if (rv && n < ncount) {
        long long off = rowoff + (long long)(n / p.n_group) * p.out_sg + (n % p.n_group);
        if (p.res) v = p.res[off] + (p.res_scale ? __ldg(p.res_scale + n) : 1.f) * v;
        a.y[off] = v;
        s1 += v;
        s2 += v * v;
      }
    }
    if (p.stats) {
      // Reduce over the 16 threads that share this output row (lanes differing in bits 0-3).
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) {
        s1 += __shfl_xor_sync(0xffffffffu, s1, o);
        s2 += __shfl_xor_sync(0xffffffffu, s2, o);
      }
      if (tx == 0 && rv) {
        int g = p.stats_per_h ? ob * p.h_out + oho : ob;
        atomicAdd(p.stats + 2 * g, (double)s1);
        atomicAdd(p.stats + 2 * g + 1, (double)s2);
      }
    }
  }
}

// Wide-tile form for channels-last inputs whose channel count is a multiple of 16 (no
// prologue): a 128 x 128 output tile per block, 8 x 8 per thread (one float4 pair of A and
// of B per k feeds 64 FMAs), and since a 16-wide K tile then lies inside one tap, each
// thread computes its input row's offset once per K tile and loads 2 float4 of channels.
// The K order of every output's sum is the generic kernel's (bit-identical results).
constexpr int WBM = 128, WBN = 128, WBK = 16, WNT = 256;

__global__ void __launch_bounds__(WNT, 2) conv_simt_wide_kernel(ConvArgs a) {
  const UnblendConvParams& p = a.p;
  __shared__ __align__(16) float As[2][WBK][WBM + 4];
  __shared__ __align__(16) float Bs[2][WBK][WBN + 4];
  const int tid = threadIdx.x;
  const long long m0 = (long long)blockIdx.x * WBM;
  const int n0 = blockIdx.y * WBN;
  // Load role: row / channel tid >> 1, K half (tid & 1) * 8.
  const int lr = tid >> 1, lk = (tid & 1) * 8;
  const long long m = m0 + lr;
  const bool mvalid = m < a.M;
  int wo = 0, ho = 0, b = 0;
  if (mvalid) {
    wo = (int)(m % p.w_out);
    const long long t = m / p.w_out;
    ho = (int)(t % p.h_out);
    b = (int)(t / p.h_out);
  }
  const int hbase = ho * p.sh - p.ph, wbase = wo * p.sw - p.pw;
  const float* xb = a.x + (long long)b * p.in_sb;
  const int nrow = n0 + lr;
  const float* wrow = a.w + (long long)nrow * a.K + lk;
  float4 ra0, ra1, rb0, rb1;
  auto load_tiles = [&](int k0) {
    const int tap = k0 / p.c_in, ci = k0 - tap * p.c_in + lk;
    const int kh = tap / p.kw, kw = tap - kh * p.kw;
    const int hi = hbase + kh * p.dh, wi = wbase + kw * p.dw;
    ra0 = ra1 = make_float4(0.f, 0.f, 0.f, 0.f);
    if (mvalid && hi >= 0 && hi < p.h_in && wi >= 0 && wi < p.w_in) {
      const float4* src = reinterpret_cast<const float4*>(xb + (long long)hi * p.in_sh + (long long)wi * p.in_sw + ci);
      ra0 = __ldg(src);
      ra1 = __ldg(src + 1);
    }
    rb0 = rb1 = make_float4(0.f, 0.f, 0.f, 0.f);
    if (nrow < p.n_out) {
      const float4* src = reinterpret_cast<const float4*>(wrow + k0);
      rb0 = __ldg(src);
      rb1 = __ldg(src + 1);
    }
  };
  auto store_tiles = [&](int buf) {
    const float av[8] = {ra0.x, ra0.y, ra0.z, ra0.w, ra1.x, ra1.y, ra1.z, ra1.w};
    const float bv[8] = {rb0.x, rb0.y, rb0.z, rb0.w, rb1.x, rb1.y, rb1.z, rb1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      As[buf][lk + i][lr] = av[i];
      Bs[buf][lk + i][lr] = bv[i];
    }
  };
  const int tx = tid & 15;  // N: 8 columns each
  const int ty = tid >> 4;  // M: 8 rows each
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  const int ktiles = a.K / WBK;
  load_tiles(0);
  store_tiles(0);
  __syncthreads();
  for (int kt = 0; kt < ktiles; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < ktiles) load_tiles((kt + 1) * WBK);
#pragma unroll
    for (int kk = 0; kk < WBK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 8]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 8 + 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 8]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 8 + 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (kt + 1 < ktiles) store_tiles(buf ^ 1);
    __syncthreads();
  }
  // Epilogue: as the generic kernel, eight columns per thread.
  const bool glu = p.act == UNBLEND_ACT_GLU;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const long long mm = m0 + ty * 8 + i;
    const bool rv = mm < a.M;
    int owo = 0, oho = 0, ob = 0;
    if (rv) {
      owo = (int)(mm % p.w_out);
      const long long t = mm / p.w_out;
      oho = (int)(t % p.h_out);
      ob = (int)(t / p.h_out);
    }
    const long long rowoff = (long long)ob * p.out_sb + (long long)oho * p.out_sh + (long long)owo * p.out_sw;
    float s1 = 0.f, s2 = 0.f;
    float vals[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int n = n0 + tx * 8 + j;
      float v = acc[i][j];
      if (n < p.n_out && a.bias) v += __ldg(a.bias + n);
      if (p.act == UNBLEND_ACT_GELU) v = ub::gelu_erf(v);
      vals[j] = v;
    }
    const int nouts = glu ? 4 : 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j >= nouts) break;
      const int n = glu ? (n0 + tx * 8) / 2 + j : n0 + tx * 8 + j;
      const int ncount = glu ? p.n_out / 2 : p.n_out;
      float v = glu ? vals[2 * j] * ub::sigmoid_approx(vals[2 * j + 1]) : vals[j];
      if (rv && n < ncount) {
        const long long off = rowoff + (long long)(n / p.n_group) * p.out_sg + (n % p.n_group);
        if (p.res) v = p.res[off] + (p.res_scale ? __ldg(p.res_scale + n) : 1.f) * v;
        a.y[off] = v;
        s1 += v;
        s2 += v * v;
      }
    }
    if (p.stats) {
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) {
        s1 += __shfl_xor_sync(0xffffffffu, s1, o);
        s2 += __shfl_xor_sync(0xffffffffu, s2, o);
      }
      if (tx == 0 && rv) {
        const int g = p.stats_per_h ? ob * p.h_out + oho : ob;
        atomicAdd(p.stats + 2 * g, (double)s1);
        atomicAdd(p.stats + 2 * g + 1, (double)s2);
      }
    }
  }
}

// First-layer convolutions (c_in <= 4 input channels, up to 8 taps along one
// axis, n_out a multiple of 16 up to 64, bias + optional GELU, nothing else):
// K = taps * c_in <= 32 is too short for the tiled kernel above, whose tile
// loads and index arithmetic then dominate. Here each thread gathers the K
// inputs of TH_PPT output positions into registers once and sweeps the output
// channels 16 at a time against the weights held transposed in shared memory
// (one broadcast float4 read feeds 4 * TH_PPT FMAs).
constexpr int TH_NT = 128;
constexpr int TH_PPT = 2;

template <int CIN, int TAPS>
__global__ void __launch_bounds__(TH_NT) conv_thin_kernel(ConvArgs a) {
  constexpr int K = CIN * TAPS;
  const UnblendConvParams& p = a.p;
  __shared__ __align__(16) float ws[K * 64];  // [k][n]
  const int N = p.n_out;
  for (int i = threadIdx.x; i < N * K; i += TH_NT) {
    const int n = i / K, k = i - n * K;
    ws[k * N + n] = __ldg(a.w + i);
  }
  const bool along_h = p.kw == 1;
  float xin[TH_PPT][K];
  long long rowoff[TH_PPT];
  bool valid[TH_PPT];
#pragma unroll
  for (int q = 0; q < TH_PPT; ++q) {
    const long long m = (long long)blockIdx.x * (TH_NT * TH_PPT) + q * TH_NT + threadIdx.x;
    valid[q] = m < a.M;
    int wo = 0, ho = 0, b = 0;
    if (valid[q]) {
      wo = (int)(m % p.w_out);
      const long long t = m / p.w_out;
      ho = (int)(t % p.h_out);
      b = (int)(t / p.h_out);
    }
    rowoff[q] = (long long)b * p.out_sb + (long long)ho * p.out_sh + (long long)wo * p.out_sw;
    const int h0 = ho * p.sh - p.ph, w0 = wo * p.sw - p.pw;
#pragma unroll
    for (int t = 0; t < TAPS; ++t) {
      const int hi = along_h ? h0 + t : h0, wi = along_h ? w0 : w0 + t;
      const bool inb = valid[q] && hi >= 0 && hi < p.h_in && wi >= 0 && wi < p.w_in;
      const float* src = a.x + (long long)b * p.in_sb + (long long)hi * p.in_sh + (long long)wi * p.in_sw;
#pragma unroll
      for (int c = 0; c < CIN; ++c) xin[q][t * CIN + c] = inb ? __ldg(src + c) : 0.f;
    }
  }
  __syncthreads();
  for (int n0 = 0; n0 < N; n0 += 16) {
    float acc[TH_PPT][16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float bj = a.bias ? __ldg(a.bias + n0 + j) : 0.f;
#pragma unroll
      for (int q = 0; q < TH_PPT; ++q) acc[q][j] = bj;
    }
#pragma unroll
    for (int k = 0; k < K; ++k) {
#pragma unroll
      for (int j4 = 0; j4 < 4; ++j4) {
        const float4 w4 = *reinterpret_cast<const float4*>(ws + k * N + n0 + 4 * j4);
#pragma unroll
        for (int q = 0; q < TH_PPT; ++q) {
          acc[q][4 * j4] = fmaf(xin[q][k], w4.x, acc[q][4 * j4]);
          acc[q][4 * j4 + 1] = fmaf(xin[q][k], w4.y, acc[q][4 * j4 + 1]);
          acc[q][4 * j4 + 2] = fmaf(xin[q][k], w4.z, acc[q][4 * j4 + 2]);
          acc[q][4 * j4 + 3] = fmaf(xin[q][k], w4.w, acc[q][4 * j4 + 3]);
        }
      }
    }
#pragma unroll
    for (int q = 0; q < TH_PPT; ++q) {
      if (!valid[q]) continue;
      float* dst = a.y + rowoff[q] + n0;
#pragma unroll
      for (int j4 = 0; j4 < 4; ++j4) {
        float4 v = make_float4(acc[q][4 * j4], acc[q][4 * j4 + 1], acc[q][4 * j4 + 2], acc[q][4 * j4 + 3]);
        if (p.act == UNBLEND_ACT_GELU) {
          v.x = ub::gelu_erf(v.x);
          v.y = ub::gelu_erf(v.y);
          v.z = ub::gelu_erf(v.z);
          v.w = ub::gelu_erf(v.w);
        }
        *reinterpret_cast<float4*>(dst + 4 * j4) = v;
      }
    }
  }
}

}  // namespace

extern "C" int unblend_conv2d_f32(const float* x, const float* w, const float* bias, float* y,
                                  const UnblendConvParams* p, void* stream) {
  UB_REQUIRE(x && w && y && p);
  UB_REQUIRE(!p->post && !p->y_bf16);  // tensor-core epilogue features
  UB_REQUIRE(p->batch > 0 && p->h_out > 0 && p->w_out > 0 && p->n_out > 0 && p->c_in > 0);
  UB_REQUIRE(p->kh > 0 && p->kw > 0 && p->sh > 0 && p->sw > 0 && p->dh > 0 && p->dw > 0);
  UB_REQUIRE(p->n_group > 0);
  UB_REQUIRE(p->act != UNBLEND_ACT_GLU || (p->n_out % 2) == 0);
  UB_REQUIRE(p->prologue != UNBLEND_PRO_GN_GELU || (p->pro_stats && p->pro_gamma && p->pro_beta));
  UB_REQUIRE(p->prologue != UNBLEND_PRO_ADD || p->pro_x2);
  ConvArgs a;
  a.p = *p;
  a.x = x;
  a.w = w;
  a.bias = bias;
  a.y = y;
  a.M = (long long)p->batch * p->h_out * p->w_out;
  a.K = p->kh * p->kw * p->c_in;
  const int taps = p->kh * p->kw;
  const bool thin = p->c_in <= 4 && (p->kh == 1 || p->kw == 1) && taps == 8 && p->dh == 1 && p->dw == 1 &&
                    p->prologue == UNBLEND_PRO_NONE && (p->act == UNBLEND_ACT_NONE || p->act == UNBLEND_ACT_GELU) &&
                    !p->res && !p->stats && p->n_out % 16 == 0 && p->n_out <= 64 && p->n_group >= p->n_out &&
                    p->out_sb % 4 == 0 && p->out_sh % 4 == 0 && p->out_sw % 4 == 0 &&
                    (reinterpret_cast<uintptr_t>(y) & 15) == 0 && (p->c_in == 1 || p->c_in == 2 || p->c_in == 4);
  if (thin) {
    const long long blocks = (a.M + TH_NT * TH_PPT - 1) / (TH_NT * TH_PPT);
    UB_REQUIRE(blocks < (1LL << 31));
    if (p->c_in == 4) conv_thin_kernel<4, 8><<<(unsigned)blocks, TH_NT, 0, ub::as_stream(stream)>>>(a);
    else if (p->c_in == 2) conv_thin_kernel<2, 8><<<(unsigned)blocks, TH_NT, 0, ub::as_stream(stream)>>>(a);
    else conv_thin_kernel<1, 8><<<(unsigned)blocks, TH_NT, 0, ub::as_stream(stream)>>>(a);
    UB_CHECK_LAUNCH();
    return 0;
  }
  const bool wide = p->prologue == UNBLEND_PRO_NONE && p->c_in % WBK == 0 && p->in_sw == p->c_in &&
                    p->in_sh % 4 == 0 && p->in_sb % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(w) & 15) == 0 && p->n_out >= 64;
  if (wide) {
    dim3 gw((unsigned)((a.M + WBM - 1) / WBM), (unsigned)((p->n_out + WBN - 1) / WBN));
    UB_REQUIRE(gw.y < 65536 && gw.x < (1u << 31));
    conv_simt_wide_kernel<<<gw, WNT, 0, ub::as_stream(stream)>>>(a);
    UB_CHECK_LAUNCH();
    return 0;
  }
  dim3 grid((unsigned)((a.M + BM - 1) / BM), (unsigned)((p->n_out + BN - 1) / BN));
  UB_REQUIRE(grid.y < 65536);
  conv_simt_kernel<<<grid, NT, 0, ub::as_stream(stream)>>>(a);
  UB_CHECK_LAUNCH();
  return 0;
}
