// SCNet kernels (unblend/scnet.py): what the sparse-compression network needs
// beyond the convolution, GroupNorm and STFT kernels it shares with the other
// models. Activations are channels-last [B, F, T, C] (frequency rows, frames,
// channels), fp32.
//
//   pad_tail        zero padding of the segment to the STFT length (stft_padding)
//   swap_axes       [B, n1, n2, G*4] -> [G, B, n2, n1, 4]: frame-major STFT output to
//                   frequency-major activations (plus the masked variant's frequency
//                   embedding), and the decoder output to per-stem iSTFT input
//   depthwise3      ConvolutionModule's depthwise conv (k = 3 along frames) with the
//                   GroupNorm(1) sums of each (batch, frequency) row
//   act_copy        strided copy with GELU / tanh / Swish (band outputs into the full
//                   band, transposed-conv trims, the mask head's tanh)
//   rfft_time / irfft_time   FeatureConversion: orthonormal real DFT along frames (mixed-radix
//                            FFTs when the frame count factors into radices up to 17, else direct sums)
//   lstm_recurrence the bidirectional LSTM recurrence of DualPathRNN (input
//                   projections precomputed by a GEMM): a thread-block cluster per 64
//                   sequences and direction with W_hh resident in shared memory for
//                   hidden sizes up to 256, W_hh streamed from L2 for 512
#include <math.h>

#include "common.cuh"

namespace {

__global__ void pad_tail_kernel(const float* __restrict__ x, float* __restrict__ y, int rows, long long n_in,
                                long long n_out) {
  const long long total = (long long)rows * n_out;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / n_out, j = i - r * n_out;
    y[i] = j < n_in ? __ldg(x + r * n_in + j) : 0.f;
  }
}

// Block (32, 8): a 32 x 32 tile of float4 elements of one (batch, group).
__global__ void swap_axes_kernel(const float4* __restrict__ x, float4* __restrict__ y, const float* __restrict__ add,
                                 int batch, int n1, int n2, int groups) {
  __shared__ float4 tile[32][33];
  const int j0 = blockIdx.x * 32, i0 = blockIdx.y * 32;
  const int b = blockIdx.z % batch, g = blockIdx.z / batch;
  for (int di = threadIdx.y; di < 32; di += 8) {
    const int i = i0 + di, j = j0 + threadIdx.x;
    if (i < n1 && j < n2) tile[di][threadIdx.x] = x[(((long long)b * n1 + i) * n2 + j) * groups + g];
  }
  __syncthreads();
  for (int dj = threadIdx.y; dj < 32; dj += 8) {
    const int j = j0 + dj, i = i0 + threadIdx.x;
    if (i < n1 && j < n2) {
      float4 v = tile[threadIdx.x][dj];
      if (add) {
        const float* a = add + (long long)(4 * g) * n2 + j;
        v.x += __ldg(a);
        v.y += __ldg(a + n2);
        v.z += __ldg(a + 2LL * n2);
        v.w += __ldg(a + 3LL * n2);
      }
      y[(((long long)g * batch + b) * n2 + j) * n1 + i] = v;
    }
  }
}

// One block per row r: u[r, t, c] = b[c] + sum_k w[c, k] z[r, t + k - 1, c] (zero outside
// [0, T)); stats[2r], stats[2r+1] = sum u, sum u^2 over the row (double).
__global__ void depthwise3_kernel(const float* __restrict__ z, const float* __restrict__ w,
                                  const float* __restrict__ bias, float* __restrict__ u, double* __restrict__ stats,
                                  int t_len, int c) {
  const long long r = blockIdx.x;
  const float* zr = z + r * t_len * (long long)c;
  float* ur = u + r * t_len * (long long)c;
  const int n = t_len * c;
  double s1 = 0.0, s2 = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int t = i / c, ch = i - t * c;
    float v = __ldg(bias + ch);
    v = fmaf(__ldg(w + 3 * ch + 1), zr[i], v);
    if (t > 0) v = fmaf(__ldg(w + 3 * ch), zr[i - c], v);
    if (t + 1 < t_len) v = fmaf(__ldg(w + 3 * ch + 2), zr[i + c], v);
    ur[i] = v;
    s1 += v;
    s2 += (double)v * v;
  }
  __shared__ double red[2][32];
  s1 = ub::warp_sum_d(s1);
  s2 = ub::warp_sum_d(s2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    red[0][warp] = s1;
    red[1][warp] = s2;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double a = 0.0, bq = 0.0;
    for (int k = 0; k < (int)(blockDim.x >> 5); ++k) {
      a += red[0][k];
      bq += red[1][k];
    }
    stats[2 * r] = a;
    stats[2 * r + 1] = bq;
  }
}

__device__ __forceinline__ float apply_act(float v, int act) {
  if (act == UNBLEND_ACT_GELU) return ub::gelu_erf(v);
  if (act == UNBLEND_ACT_TANH) return tanhf(v);
  if (act == UNBLEND_ACT_SWISH) return v / (1.0f + expf(-v));
  return v;
}

__global__ void act_copy_kernel(const float* __restrict__ x, long long xs, float* __restrict__ y, long long ys,
                                int count, long long n, int act) {
  const long long total = (long long)count * n;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long k = i / n, j = i - k * n;
    y[k * ys + j] = apply_act(x[k * xs + j], act);
  }
}

// cos / sin of 2 pi j / T for j < T, from double precision, in shared memory.
__device__ __forceinline__ void twiddle_table(float2* tab, int t_len) {
  for (int j = threadIdx.x; j < t_len; j += blockDim.x) {
    double s, c;
    sincospi(2.0 * (double)j / (double)t_len, &s, &c);
    tab[j] = make_float2((float)c, (float)s);
  }
}

// Grid (rows, ceil(C / 32)), 256 threads. x [rows, T, C] -> y [rows, K, 2C], K = T/2 + 1:
// y[., k, c] = sum_t x[t, c] cos(2 pi k t / T) / sqrt(T), y[., k, C + c] = -sum_t x sin(...) / sqrt(T).
// Lane = channel of the 32-channel slice; warp w computes bins w, w + 8, ... four at a time.
__global__ void __launch_bounds__(256) rfft_time_kernel(const float* __restrict__ x, float* __restrict__ y, int t_len,
                                                        int c) {
  extern __shared__ __align__(16) float sm[];
  float2* tab = reinterpret_cast<float2*>(sm);
  float* xs = sm + 2 * t_len;  // [T][32]
  const long long r = blockIdx.x;
  const int c0 = blockIdx.y * 32, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nk = t_len / 2 + 1;
  twiddle_table(tab, t_len);
  for (int i = threadIdx.x; i < t_len * 32; i += blockDim.x) {
    const int t = i >> 5, ch = c0 + (i & 31);
    xs[i] = ch < c ? __ldg(x + (r * t_len + t) * c + ch) : 0.f;
  }
  __syncthreads();
  const float scale = rsqrtf((float)t_len);
  const int ch = c0 + lane;
  for (int kb = warp; kb < nk; kb += 32) {
    float re[4] = {0.f, 0.f, 0.f, 0.f}, im[4] = {0.f, 0.f, 0.f, 0.f};
    int idx[4] = {0, 0, 0, 0}, kk[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) kk[q] = kb + 8 * q < nk ? kb + 8 * q : 0;
    for (int t = 0; t < t_len; ++t) {
      const float v = xs[t * 32 + lane];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 w = tab[idx[q]];
        re[q] = fmaf(v, w.x, re[q]);
        im[q] = fmaf(-v, w.y, im[q]);
        idx[q] += kk[q];
        if (idx[q] >= t_len) idx[q] -= t_len;
      }
    }
    if (ch < c) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int k = kb + 8 * q;
        if (k < nk) {
          float* o = y + (r * nk + k) * 2LL * c;
          o[ch] = re[q] * scale;
          o[c + ch] = im[q] * scale;
        }
      }
    }
  }
}

// Grid (rows, ceil(C / 32)), 256 threads. y [rows, K, 2C] -> x [rows, T, C], T = 2 (K - 1):
// x[t, c] = (Re y_0 + (-1)^t Re y_{K-1} + 2 sum_{0<k<K-1} (Re y_k cos - Im y_k sin)(2 pi k t / T)) / sqrt(T)
// (the imaginary parts of the first and last bins do not enter a real inverse transform).
__global__ void __launch_bounds__(256) irfft_time_kernel(const float* __restrict__ y, float* __restrict__ x, int nk,
                                                         int c) {
  extern __shared__ __align__(16) float sm[];
  const int t_len = 2 * (nk - 1);
  float2* tab = reinterpret_cast<float2*>(sm);
  float* re_s = sm + 2 * t_len;   // [K][32]
  float* im_s = re_s + nk * 32;   // [K][32]
  const long long r = blockIdx.x;
  const int c0 = blockIdx.y * 32, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  twiddle_table(tab, t_len);
  for (int i = threadIdx.x; i < nk * 32; i += blockDim.x) {
    const int k = i >> 5, ch = c0 + (i & 31);
    const float* src = y + (r * nk + k) * 2LL * c;
    const bool edge = k == 0 || k == nk - 1;
    re_s[i] = ch < c ? (edge ? 1.f : 2.f) * __ldg(src + ch) : 0.f;
    im_s[i] = ch < c && !edge ? 2.f * __ldg(src + c + ch) : 0.f;
  }
  __syncthreads();
  const float scale = rsqrtf((float)t_len);
  const int ch = c0 + lane;
  for (int tb = warp; tb < t_len; tb += 32) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int idx[4] = {0, 0, 0, 0}, tt[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) tt[q] = tb + 8 * q < t_len ? tb + 8 * q : 0;
    for (int k = 0; k < nk; ++k) {
      const float a = re_s[k * 32 + lane], bq = im_s[k * 32 + lane];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 w = tab[idx[q]];
        acc[q] = fmaf(a, w.x, acc[q]);
        acc[q] = fmaf(-bq, w.y, acc[q]);
        idx[q] += tt[q];
        if (idx[q] >= t_len) idx[q] -= t_len;
      }
    }
    if (ch < c) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int t = tb + 8 * q;
        if (t < t_len) x[(r * t_len + t) * (long long)c + ch] = acc[q] * scale;
      }
    }
  }
}

// Bidirectional LSTM recurrence (torch.nn.LSTM, gates i, f, g, o):
//   g = xp[seq, step] + W_hh h_prev;  c = s(f) c + s(i) tanh(g_g);  h = s(o) tanh(c)
// Grid (ceil(n_seq / (P * G)), 2 directions), 256 threads. P = 256 / min(H, 256) parts
// of the block each run G sequences; a thread owns U = max(1, H / 256) hidden units of
// its part. xp rows hold [forward 4H | reverse 4H] gate pre-activations (input
// projection and both biases); whh_t[dir] is W_hh transposed, [H][4H]; h_out rows
// receive [forward H | reverse H]. Row of (seq, step): (seq / inner) * outer_stride +
// (seq % inner) * inner_stride + step * step_stride.
template <int G, int U>
__global__ void __launch_bounds__(256) lstm_recurrence_kernel(const float* __restrict__ xp,
                                                              const float* __restrict__ whh_t,
                                                              float* __restrict__ h_out, int n_seq, int steps, int hid,
                                                              int inner, long long outer_stride,
                                                              long long inner_stride, long long step_stride) {
  extern __shared__ __align__(16) float hbuf[];  // [2][P][H][G]
  const int dir = blockIdx.y;
  const int tpp = hid < 256 ? hid : 256;  // threads per part
  const int parts = 256 / tpp;
  const int part = threadIdx.x / tpp, tl = threadIdx.x - part * tpp;
  const int seq0 = (blockIdx.x * parts + part) * G;
  const float* w = whh_t + (long long)dir * hid * 4 * hid;
  long long rowb[G];
  bool live[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int s = seq0 + g;
    live[g] = s < n_seq;
    const int sq = live[g] ? s : 0;
    rowb[g] = (long long)(sq / inner) * outer_stride + (long long)(sq % inner) * inner_stride;
  }
  float cst[U][G];
#pragma unroll
  for (int m = 0; m < U; ++m)
#pragma unroll
    for (int g = 0; g < G; ++g) cst[m][g] = 0.f;
  float* hpart[2] = {hbuf + (long long)part * hid * G, hbuf + ((long long)parts + part) * hid * G};
  for (int i = tl; i < hid * G; i += tpp) hpart[0][i] = 0.f;
  __syncthreads();
  const long long xs = 8LL * hid, hs = 2LL * hid;
  for (int it = 0; it < steps; ++it) {
    const int step = dir == 0 ? it : steps - 1 - it;
    const float* hcur = hpart[it & 1];
    float* hnext = hpart[(it + 1) & 1];
    float acc[U][4][G];
#pragma unroll
    for (int m = 0; m < U; ++m) {
      const int u = tl + m * tpp;
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int g = 0; g < G; ++g)
          acc[m][q][g] = live[g] ? __ldg(xp + (rowb[g] + step * step_stride) * xs + dir * 4LL * hid + q * hid + u)
                                 : 0.f;
    }
#pragma unroll 2
    for (int k = 0; k < hid; ++k) {
      float hv[G];
#pragma unroll
      for (int g4 = 0; g4 < G; g4 += 4) {
        const float4 v = *reinterpret_cast<const float4*>(hcur + k * G + g4);
        hv[g4] = v.x;
        hv[g4 + 1] = v.y;
        hv[g4 + 2] = v.z;
        hv[g4 + 3] = v.w;
      }
      const float* wk = w + (long long)k * 4 * hid;
#pragma unroll
      for (int m = 0; m < U; ++m) {
        const int u = tl + m * tpp;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float wv = __ldg(wk + q * hid + u);
#pragma unroll
          for (int g = 0; g < G; ++g) acc[m][q][g] = fmaf(wv, hv[g], acc[m][q][g]);
        }
      }
    }
#pragma unroll
    for (int m = 0; m < U; ++m) {
      const int u = tl + m * tpp;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float ig = 1.0f / (1.0f + expf(-acc[m][0][g]));
        const float fg = 1.0f / (1.0f + expf(-acc[m][1][g]));
        const float gg = tanhf(acc[m][2][g]);
        const float og = 1.0f / (1.0f + expf(-acc[m][3][g]));
        cst[m][g] = fg * cst[m][g] + ig * gg;
        const float h = og * tanhf(cst[m][g]);
        hnext[u * G + g] = h;
        if (live[g]) h_out[(rowb[g] + step * step_stride) * hs + dir * (long long)hid + u] = h;
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Real DFTs along frames as mixed-radix FFTs (radices 2, 3, 4, 5, 7, 11, 13, 17; 476
// frames = 4 x 7 x 17). A block takes FFT_PAIRS channel pairs of one row; channels
// (2p, 2p + 1) travel as the real and imaginary parts of one complex sequence, so one
// complex FFT serves two real transforms. Each stage is one pass of the Stockham
// autosort formulation (Govindaraju et al., "High performance discrete Fourier
// transforms on graphics processors", SC 2008): butterfly j of a radix-R stage with Ns
// already combined points reads in[j + r T / R] (r < R), rotates element r by the
// twiddle of (j mod Ns) r / (Ns R) turns, takes an R-point DFT and writes
// out[(j / Ns) Ns R + (j mod Ns) + r Ns]; the output is in natural order. Twiddles come
// from a table of cos / sin (2 pi i / T) evaluated in double precision.
constexpr int FFT_PAIRS = 8;     // channel pairs per block (16 channels)
constexpr int FFT_THREADS = 256; // FFT_PAIRS pairs x 32 butterfly workers
constexpr int FFT_MAXR = 8;      // radices per factorisation

struct FftPlan {
  int n;
  int radix[FFT_MAXR];
};

// e^{sign 2 pi i idx / T} from the table (tab[i] = (cos, sin) of 2 pi i / T).
__device__ __forceinline__ float2 tw(const float2* tab, int idx, float sign) {
  const float2 w = tab[idx];
  return make_float2(w.x, sign * w.y);
}

__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}

template <int R>
__device__ __forceinline__ void fft_stage(const float2* __restrict__ in, float2* __restrict__ out, int T, int ns,
                                          const float2* __restrict__ tab, float sign, int pair, int worker) {
  const int m = T / R, step_r = T / R;  // butterflies per pair; table stride of 1 / R turn
  for (int j = worker; j < m; j += FFT_THREADS / FFT_PAIRS) {
    const int k = j % ns;
    float2 v[R];
#pragma unroll
    for (int r = 0; r < R; ++r) v[r] = in[(j + r * m) * FFT_PAIRS + pair];
    if (ns > 1) {
      const int unit = T / (ns * R);  // table stride of 1 / (ns R) turn
#pragma unroll
      for (int r = 1; r < R; ++r) v[r] = cmul(v[r], tw(tab, k * r * unit, sign));
    }
    float2 o[R];
#pragma unroll
    for (int q = 0; q < R; ++q) {
      float2 acc = v[0];
#pragma unroll
      for (int r = 1; r < R; ++r) {
        const float2 w = tw(tab, ((r * q) % R) * step_r, sign);
        acc.x = fmaf(v[r].x, w.x, fmaf(-v[r].y, w.y, acc.x));
        acc.y = fmaf(v[r].x, w.y, fmaf(v[r].y, w.x, acc.y));
      }
      o[q] = acc;
    }
    const int base = (j / ns) * ns * R + k;
#pragma unroll
    for (int q = 0; q < R; ++q) out[(base + q * ns) * FFT_PAIRS + pair] = o[q];
  }
}

// In-place over the two buffers: the result ends in buf[0] or buf[1] (returned).
__device__ float2* fft_run(float2* a, float2* b, const FftPlan& plan, const float2* tab, float sign, int pair,
                           int worker) {
  int ns = 1;
  for (int s = 0; s < FFT_MAXR && plan.radix[s] > 1; ++s) {
    const int R = plan.radix[s];
    switch (R) {
      case 2: fft_stage<2>(a, b, plan.n, ns, tab, sign, pair, worker); break;
      case 3: fft_stage<3>(a, b, plan.n, ns, tab, sign, pair, worker); break;
      case 4: fft_stage<4>(a, b, plan.n, ns, tab, sign, pair, worker); break;
      case 5: fft_stage<5>(a, b, plan.n, ns, tab, sign, pair, worker); break;
      case 7: fft_stage<7>(a, b, plan.n, ns, tab, sign, pair, worker); break;
      case 11: fft_stage<11>(a, b, plan.n, ns, tab, sign, pair, worker); break;
      case 13: fft_stage<13>(a, b, plan.n, ns, tab, sign, pair, worker); break;
      default: fft_stage<17>(a, b, plan.n, ns, tab, sign, pair, worker); break;
    }
    __syncthreads();
    ns *= R;
    float2* t = a;
    a = b;
    b = t;
  }
  return a;
}

// Grid (rows, ceil(C / 16)). x [rows, T, C] -> y [rows, K, 2C] (K = T/2 + 1), orthonormal:
// y[., k, c] = Re X_c[k] / sqrt(T), y[., k, C + c] = Im X_c[k] / sqrt(T), X = sum_t x e^{-2 pi i k t / T}.
__global__ void __launch_bounds__(FFT_THREADS) rfft_fft_kernel(const float* __restrict__ x, float* __restrict__ y,
                                                              int C, const FftPlan plan) {
  extern __shared__ __align__(16) float2 fsm[];
  const int T = plan.n, K = T / 2 + 1;
  float2* tab = fsm;
  float2* a = fsm + T;
  float2* b = a + T * FFT_PAIRS;
  const long long row = blockIdx.x;
  const int pair = threadIdx.x % FFT_PAIRS, worker = threadIdx.x / FFT_PAIRS;
  const int ch0 = blockIdx.y * 2 * FFT_PAIRS + 2 * pair, ch1 = ch0 + 1;
  twiddle_table(tab, T);
  for (int t = worker; t < T; t += FFT_THREADS / FFT_PAIRS) {
    const float* xr = x + (row * T + t) * C;
    a[t * FFT_PAIRS + pair] = make_float2(ch0 < C ? __ldg(xr + ch0) : 0.f, ch1 < C ? __ldg(xr + ch1) : 0.f);
  }
  __syncthreads();
  const float2* z = fft_run(a, b, plan, tab, -1.f, pair, worker);
  const float s = rsqrtf((float)T);
  for (int k = worker; k < K; k += FFT_THREADS / FFT_PAIRS) {
    const float2 p = z[k * FFT_PAIRS + pair], q = z[((T - k) % T) * FFT_PAIRS + pair];
    // Channel ch0 = (Z[k] + conj Z[T-k]) / 2, ch1 = (Z[k] - conj Z[T-k]) / 2i.
    float* yr = y + (row * K + k) * 2LL * C;
    if (ch0 < C) {
      yr[ch0] = 0.5f * (p.x + q.x) * s;
      yr[C + ch0] = 0.5f * (p.y - q.y) * s;
    }
    if (ch1 < C) {
      yr[ch1] = 0.5f * (p.y + q.y) * s;
      yr[C + ch1] = -0.5f * (p.x - q.x) * s;
    }
  }
}

// Grid (rows, ceil(C / 16)). y [rows, K, 2C] -> x [rows, T, C], T = 2 (K - 1): the inverse of the
// Hermitian spectrum (imaginary parts of bins 0 and K - 1 dropped), orthonormal.
__global__ void __launch_bounds__(FFT_THREADS) irfft_fft_kernel(const float* __restrict__ y, float* __restrict__ x,
                                                               int C, const FftPlan plan) {
  extern __shared__ __align__(16) float2 fsm[];
  const int T = plan.n, K = T / 2 + 1;
  float2* tab = fsm;
  float2* a = fsm + T;
  float2* b = a + T * FFT_PAIRS;
  const long long row = blockIdx.x;
  const int pair = threadIdx.x % FFT_PAIRS, worker = threadIdx.x / FFT_PAIRS;
  const int ch0 = blockIdx.y * 2 * FFT_PAIRS + 2 * pair, ch1 = ch0 + 1;
  twiddle_table(tab, T);
  for (int k = worker; k < T; k += FFT_THREADS / FFT_PAIRS) {
    const int kk = k < K ? k : T - k;  // bins past K - 1 are conjugates of T - k
    const float* yr = y + (row * K + kk) * 2LL * C;
    const bool keep_im = kk != 0 && kk != K - 1;
    float2 sa = make_float2(ch0 < C ? __ldg(yr + ch0) : 0.f, ch0 < C && keep_im ? __ldg(yr + C + ch0) : 0.f);
    float2 sb = make_float2(ch1 < C ? __ldg(yr + ch1) : 0.f, ch1 < C && keep_im ? __ldg(yr + C + ch1) : 0.f);
    if (k >= K) {
      sa.y = -sa.y;
      sb.y = -sb.y;
    }
    a[k * FFT_PAIRS + pair] = make_float2(sa.x - sb.y, sa.y + sb.x);  // S_a + i S_b
  }
  __syncthreads();
  const float2* z = fft_run(a, b, plan, tab, 1.f, pair, worker);
  const float s = rsqrtf((float)T);
  for (int t = worker; t < T; t += FFT_THREADS / FFT_PAIRS) {
    const float2 v = z[t * FFT_PAIRS + pair];
    float* xr = x + (row * T + t) * C;
    if (ch0 < C) xr[ch0] = v.x * s;
    if (ch1 < C) xr[ch1] = v.y * s;
  }
}

// Radices for an FFT of n points (fours first), or false when a prime factor exceeds 17
// or more than FFT_MAXR stages would be needed.
bool fft_plan(int n, FftPlan* p) {
  p->n = n;
  for (int i = 0; i < FFT_MAXR; ++i) p->radix[i] = 1;
  int s = 0;
  const int primes[] = {4, 2, 3, 5, 7, 11, 13, 17};
  for (int r : primes) {
    while (n % r == 0) {
      if (s == FFT_MAXR) return false;
      p->radix[s++] = r;
      n /= r;
    }
  }
  return n == 1;
}

// Cluster form for hid = 32 * Q <= 256: a cluster of Q CTAs runs one direction of
// G = 8 * SG sequences. CTA r of the cluster owns hidden units [32 r, 32 r + 32): their
// four gate columns of W_hh^T stay in shared memory for the whole launch (as float4
// [k][unit] = gates i, f, g, o), and every CTA keeps the h of all G sequences ([k][seq],
// double-buffered). A warp covers 8 units x 4 sequence groups of SG: per k it reads one
// float4 of W per unit (8 distinct addresses) and SG / 4 float4 of h per group (4
// distinct), both one shared-memory wavefront, for 4 SG FMAs per thread. After the k loop
// a thread updates c and h of its unit for its SG sequences, stores h and pushes it into
// the h buffer of every CTA of the cluster (distributed shared memory); one cluster
// barrier per step publishes the new h before any CTA reads it, and no CTA writes a
// buffer another may still read (step t + 1 writes the buffer read in step t, which
// every CTA finished before the barrier). The next step's input projections are loaded
// into registers before the k loop, so their latency hides behind it.
// Shared memory: 4 (128 hid + 16 SG hid) bytes.
__device__ __forceinline__ uint32_t cluster_rank_u32() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void st_cluster_v4(uint32_t local_addr, uint32_t rank, float4 v) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(remote), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}

__device__ __forceinline__ float sigmoid_f(float v) { return 1.0f / (1.0f + expf(-v)); }

// acc[q][p] += w.q * (h[2p], h[2p + 1]) for the four gates q and SG / 2 sequence pairs p,
// as packed two-lane FMAs.
template <int SG>
__device__ __forceinline__ void lstm_fma4(float2 (&acc)[4][SG / 2], const float4 w, const float4 (&h)[SG / 4]) {
#pragma unroll
  for (int h4 = 0; h4 < SG / 4; ++h4) {
    const float2 h01 = make_float2(h[h4].x, h[h4].y), h23 = make_float2(h[h4].z, h[h4].w);
    const float wq[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      acc[q][2 * h4] = ub::fma2(make_float2(wq[q], wq[q]), h01, acc[q][2 * h4]);
      acc[q][2 * h4 + 1] = ub::fma2(make_float2(wq[q], wq[q]), h23, acc[q][2 * h4 + 1]);
    }
  }
}

template <int Q, int SG>
__global__ void __launch_bounds__(256, 1) lstm_cluster_kernel(const float* __restrict__ xp,
                                                              const float* __restrict__ whh_t,
                                                              float* __restrict__ h_out, int n_seq, int steps,
                                                              int inner, long long outer_stride,
                                                              long long inner_stride, long long step_stride) {
  static_assert(SG == 4 || SG == 8, "four or eight sequences per thread");
  constexpr int HID = 32 * Q, G = 8 * SG, KU = SG == 4 ? 4 : 2;
  static_assert(HID % (2 * KU) == 0, "whole chunk pairs");
  extern __shared__ __align__(16) float sm[];
  float4* ws = reinterpret_cast<float4*>(sm);  // [HID][32]: (i, f, g, o) of this CTA's units
  float* hb = sm + HID * 128;                   // [2][HID][G]
  const uint32_t rank = cluster_rank_u32();
  const int dir = blockIdx.y;
  const int cluster = blockIdx.x / Q;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ul = (warp & 3) * 8 + (lane & 7);        // unit within the CTA
  const int sbase = ((warp >> 2) * 4 + (lane >> 3)) * SG;  // first sequence within the cluster
  const int unit = 32 * (int)rank + ul;
  const float* w = whh_t + (long long)dir * HID * 4 * HID;
  for (int i = threadIdx.x; i < HID * 128; i += 256) {
    const int k = i >> 7, r = i & 127, u = r >> 2, q = r & 3;
    sm[i] = __ldg(w + (long long)k * 4 * HID + q * HID + 32 * (int)rank + u);
  }
  for (int i = threadIdx.x; i < HID * G; i += 256) hb[i] = 0.f;
  long long rowb[SG];
  bool live[SG];
#pragma unroll
  for (int g = 0; g < SG; ++g) {
    const int s = cluster * G + sbase + g;
    live[g] = s < n_seq;
    const int sq = live[g] ? s : 0;
    rowb[g] = (long long)(sq / inner) * outer_stride + (long long)(sq % inner) * inner_stride;
  }
  float cst[SG];
#pragma unroll
  for (int g = 0; g < SG; ++g) cst[g] = 0.f;
  const long long xs = 8LL * HID, hs = 2LL * HID;
  const float* xcol = xp + dir * 4LL * HID + unit;
  float nx[4][SG];
  {
    const int step0 = dir == 0 ? 0 : steps - 1;
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int g = 0; g < SG; ++g) nx[q][g] = live[g] ? __ldg(xcol + (rowb[g] + step0 * step_stride) * xs + q * HID) : 0.f;
  }
  // Every CTA's buffers are zeroed (and its W slice loaded) before any CTA pushes h.
  cluster_sync_all();
  for (int it = 0; it < steps; ++it) {
    const int step = dir == 0 ? it : steps - 1 - it;
    const float* hcur = hb + (it & 1) * HID * G + sbase;
    float* hnext = hb + ((it + 1) & 1) * HID * G;
    float2 acc[4][SG / 2];
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int p = 0; p < SG / 2; ++p) acc[q][p] = make_float2(nx[q][2 * p], nx[q][2 * p + 1]);
    if (it + 1 < steps) {
      const int sn = dir == 0 ? it + 1 : steps - 2 - it;
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int g = 0; g < SG; ++g)
          nx[q][g] = live[g] ? __ldg(xcol + (rowb[g] + sn * step_stride) * xs + q * HID) : 0.f;
    }
    // k in chunks of KU, the shared-memory operands of the next chunk loaded into
    // registers while the current one is multiplied (two warps per scheduler cannot hide
    // the load latency otherwise).
    float4 wr0[KU], wr1[KU], hr0[KU][SG / 4], hr1[KU][SG / 4];
#pragma unroll
    for (int j = 0; j < KU; ++j) {
      wr0[j] = ws[j * 32 + ul];
#pragma unroll
      for (int h4 = 0; h4 < SG / 4; ++h4) hr0[j][h4] = *reinterpret_cast<const float4*>(hcur + j * G + 4 * h4);
    }
    for (int kc = 0; kc < HID; kc += 2 * KU) {
#pragma unroll
      for (int j = 0; j < KU; ++j) {
        wr1[j] = ws[(kc + KU + j) * 32 + ul];
#pragma unroll
        for (int h4 = 0; h4 < SG / 4; ++h4)
          hr1[j][h4] = *reinterpret_cast<const float4*>(hcur + (kc + KU + j) * G + 4 * h4);
      }
#pragma unroll
      for (int j = 0; j < KU; ++j) lstm_fma4<SG>(acc, wr0[j], hr0[j]);
      if (kc + 2 * KU < HID) {
#pragma unroll
        for (int j = 0; j < KU; ++j) {
          wr0[j] = ws[(kc + 2 * KU + j) * 32 + ul];
#pragma unroll
          for (int h4 = 0; h4 < SG / 4; ++h4)
            hr0[j][h4] = *reinterpret_cast<const float4*>(hcur + (kc + 2 * KU + j) * G + 4 * h4);
        }
      }
#pragma unroll
      for (int j = 0; j < KU; ++j) lstm_fma4<SG>(acc, wr1[j], hr1[j]);
    }
    float hn[SG];
#pragma unroll
    for (int g = 0; g < SG; ++g) {
      const float a0 = g & 1 ? acc[0][g >> 1].y : acc[0][g >> 1].x, a1 = g & 1 ? acc[1][g >> 1].y : acc[1][g >> 1].x;
      const float a2 = g & 1 ? acc[2][g >> 1].y : acc[2][g >> 1].x, a3 = g & 1 ? acc[3][g >> 1].y : acc[3][g >> 1].x;
      const float ig = sigmoid_f(a0);
      const float fg = sigmoid_f(a1);
      const float gg = tanhf(a2);
      const float og = sigmoid_f(a3);
      cst[g] = fg * cst[g] + ig * gg;
      hn[g] = og * tanhf(cst[g]);
      if (live[g]) h_out[(rowb[g] + step * step_stride) * hs + dir * (long long)HID + unit] = hn[g];
    }
    const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(hnext + unit * G + sbase));
#pragma unroll
    for (int r = 0; r < Q; ++r)
#pragma unroll
      for (int g4 = 0; g4 < SG; g4 += 4)
        st_cluster_v4(dst + 4 * g4, (uint32_t)r, make_float4(hn[g4], hn[g4 + 1], hn[g4 + 2], hn[g4 + 3]));
    cluster_sync_all();
  }
}

template <int Q, int SG>
cudaError_t launch_lstm_cluster(const float* xp, const float* whh_t, float* h_out, int n_seq, int steps, int inner,
                                long long outer_stride, long long inner_stride, long long step_stride,
                                cudaStream_t st) {
  constexpr int HID = 32 * Q, G = 8 * SG;
  const size_t smem = sizeof(float) * ((size_t)HID * 128 + 2 * (size_t)HID * G);
  cudaError_t e = cudaFuncSetAttribute(lstm_cluster_kernel<Q, SG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((n_seq + G - 1) / G) * Q, 2, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = Q;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, lstm_cluster_kernel<Q, SG>, xp, whh_t, h_out, n_seq, steps, inner, outer_stride,
                            inner_stride, step_stride);
}

}  // namespace

extern "C" int unblend_pad_tail(const float* x, float* y, int rows, long long n_in, long long n_out, void* stream) {
  UB_REQUIRE(x && y && rows > 0 && n_in > 0 && n_out >= n_in);
  pad_tail_kernel<<<ub::grid_1d((long long)rows * n_out, 256), 256, 0, ub::as_stream(stream)>>>(x, y, rows, n_in,
                                                                                               n_out);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_swap_axes(const float* x, float* y, const float* add, int batch, int n1, int n2, int groups,
                                 void* stream) {
  UB_REQUIRE(x && y && batch > 0 && n1 > 0 && n2 > 0 && groups > 0 && x != y);
  UB_REQUIRE((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0);
  UB_REQUIRE(!add || groups == 1);
  UB_REQUIRE((long long)batch * groups < 65536);
  dim3 grid((n2 + 31) / 32, (n1 + 31) / 32, batch * groups);
  swap_axes_kernel<<<grid, dim3(32, 8), 0, ub::as_stream(stream)>>>(reinterpret_cast<const float4*>(x),
                                                                    reinterpret_cast<float4*>(y), add, batch, n1, n2,
                                                                    groups);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_depthwise3(const float* z, const float* w, const float* bias, float* u, double* stats, int rows,
                                  int t_len, int c, void* stream) {
  UB_REQUIRE(z && w && bias && u && stats && rows > 0 && t_len > 0 && c > 0 && z != u);
  UB_REQUIRE(rows < (1 << 30) && (long long)t_len * c < (1LL << 31));
  depthwise3_kernel<<<rows, 256, 0, ub::as_stream(stream)>>>(z, w, bias, u, stats, t_len, c);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_act_copy(const float* x, long long x_stride, float* y, long long y_stride, int count,
                                long long n, int act, void* stream) {
  UB_REQUIRE(x && y && count > 0 && n > 0 && x_stride >= 0 && y_stride >= 0);
  UB_REQUIRE(act == UNBLEND_ACT_NONE || act == UNBLEND_ACT_GELU || act == UNBLEND_ACT_TANH ||
             act == UNBLEND_ACT_SWISH);
  UB_REQUIRE(x != y || x_stride == y_stride);
  act_copy_kernel<<<ub::grid_1d((long long)count * n, 256), 256, 0, ub::as_stream(stream)>>>(x, x_stride, y,
                                                                                           y_stride, count, n, act);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_rfft_time(const float* x, float* y, int rows, int t_len, int c, void* stream) {
  UB_REQUIRE(x && y && x != y && rows > 0 && t_len >= 2 && t_len % 2 == 0 && c > 0 && rows < (1 << 30));
  FftPlan plan;
  if (fft_plan(t_len, &plan)) {
    const size_t smem = sizeof(float2) * (size_t)t_len * (1 + 2 * FFT_PAIRS);
    UB_REQUIRE(smem <= 200 * 1024);
    cudaFuncSetAttribute(rfft_fft_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    rfft_fft_kernel<<<dim3(rows, (c + 2 * FFT_PAIRS - 1) / (2 * FFT_PAIRS)), FFT_THREADS, smem,
                      ub::as_stream(stream)>>>(x, y, c, plan);
    UB_CHECK_LAUNCH();
    return 0;
  }
  // Frame counts with a prime factor above 17: the direct sums.
  const size_t smem = sizeof(float) * (2 * (size_t)t_len + 32 * (size_t)t_len);
  UB_REQUIRE(smem <= 220 * 1024);
  cudaFuncSetAttribute(rfft_time_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  rfft_time_kernel<<<dim3(rows, (c + 31) / 32), 256, smem, ub::as_stream(stream)>>>(x, y, t_len, c);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_irfft_time(const float* y, float* x, int rows, int n_bins, int c, void* stream) {
  UB_REQUIRE(x && y && x != y && rows > 0 && n_bins >= 2 && c > 0 && rows < (1 << 30));
  const int t_len = 2 * (n_bins - 1);
  FftPlan plan;
  if (fft_plan(t_len, &plan)) {
    const size_t smem_f = sizeof(float2) * (size_t)t_len * (1 + 2 * FFT_PAIRS);
    UB_REQUIRE(smem_f <= 200 * 1024);
    cudaFuncSetAttribute(irfft_fft_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_f);
    irfft_fft_kernel<<<dim3(rows, (c + 2 * FFT_PAIRS - 1) / (2 * FFT_PAIRS)), FFT_THREADS, smem_f,
                       ub::as_stream(stream)>>>(y, x, c, plan);
    UB_CHECK_LAUNCH();
    return 0;
  }
  const size_t smem = sizeof(float) * (2 * (size_t)t_len + 64 * (size_t)n_bins);
  UB_REQUIRE(smem <= 220 * 1024);
  cudaFuncSetAttribute(irfft_time_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  irfft_time_kernel<<<dim3(rows, (c + 31) / 32), 256, smem, ub::as_stream(stream)>>>(y, x, n_bins, c);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_lstm_recurrence(const float* xp, const float* whh_t, float* h_out, int n_seq, int steps,
                                       int hid, int inner, long long outer_stride, long long inner_stride,
                                       long long step_stride, void* stream) {
  UB_REQUIRE(xp && whh_t && h_out && n_seq > 0 && steps > 0 && inner > 0);
  UB_REQUIRE(hid == 32 || hid == 64 || hid == 128 || hid == 256 || hid == 512);
  cudaStream_t st = ub::as_stream(stream);
  if (hid <= 256) {
    // A cluster of hid / 32 CTAs per 8 SG sequences and direction. Eight sequences per
    // thread halve the shared-memory reads of h per FMA; four keep more SMs busy when the
    // pass has few sequences (and are the only fit in shared memory at hid 256).
    const int q = hid / 32;
    const long long ctas8 = 2LL * q * ((n_seq + 63) / 64);
    const bool sg8 = hid < 256 && ctas8 >= 2 * 148;
    using Launch = cudaError_t (*)(const float*, const float*, float*, int, int, int, long long, long long, long long,
                                   cudaStream_t);
    const Launch launch = q == 1   ? (sg8 ? launch_lstm_cluster<1, 8> : launch_lstm_cluster<1, 4>)
                          : q == 2 ? (sg8 ? launch_lstm_cluster<2, 8> : launch_lstm_cluster<2, 4>)
                          : q == 4 ? (sg8 ? launch_lstm_cluster<4, 8> : launch_lstm_cluster<4, 4>)
                                   : launch_lstm_cluster<8, 4>;
    const cudaError_t e = launch(xp, whh_t, h_out, n_seq, steps, inner, outer_stride, inner_stride, step_stride, st);
    if (e != cudaSuccess) return (int)e;
    UB_CHECK_LAUNCH();
    return 0;
  }
  constexpr int G = 8;
  const int tpp = hid < 256 ? hid : 256;
  const int parts = 256 / tpp;
  const int per_block = parts * G;
  const unsigned blocks = (unsigned)((n_seq + per_block - 1) / per_block);
  const size_t smem = sizeof(float) * 2 * (size_t)parts * hid * G;
  if (hid <= 256) {
    cudaFuncSetAttribute(lstm_recurrence_kernel<G, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    lstm_recurrence_kernel<G, 1><<<dim3(blocks, 2), 256, smem, st>>>(xp, whh_t, h_out, n_seq, steps, hid, inner,
                                                                     outer_stride, inner_stride, step_stride);
  } else {
    cudaFuncSetAttribute(lstm_recurrence_kernel<G, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    lstm_recurrence_kernel<G, 2><<<dim3(blocks, 2), 256, smem, st>>>(xp, whh_t, h_out, n_seq, steps, hid, inner,
                                                                     outer_stride, inner_stride, step_stride);
  }
  UB_CHECK_LAUNCH();
  return 0;
}
