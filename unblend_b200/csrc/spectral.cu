// STFT front end and iSTFT output stage of HTDemucs (fp32), with an
// in-shared-memory radix-4 Stockham FFT (the autosort formulation of
// Govindaraju et al., "High performance discrete Fourier transforms on
// graphics processors", SC 2008).
//
// Front end (unblend/htdemucs.py:370-395 `_spec` + unblend/blocks.py:60-88
// `spectro`): double reflect padding, periodic Hann window, normalized STFT
// (x 1/sqrt(nfft)), Nyquist bin dropped, frames 2..2+le kept, complex as
// channels. The two audio channels of a frame share one complex FFT
// (z = x0 + i x1) and are separated with the Hermitian split.
//
// Output stage (unblend/htdemucs.py:692-704, `_ispec` :397-412,
// unblend/blocks.py:165-204 `ispectro` / torch.istft): de-normalise the CaC
// spectrogram, inverse real FFT (imaginary parts of DC and Nyquist ignored, as
// a C2R transform does), x sqrt(nfft) window, overlap-add with the squared
// window envelope of all nfft/hop + frames frames, centre crop, then add the
// de-normalised time branch.
#include "common.cuh"

namespace {

constexpr int N = 4096;
constexpr int HOP = 1024;
constexpr int NT = 256;

__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}

// Forward complex FFT of N points in shared memory (ping-pong buffers).
// tw[m] = exp(-2 pi i m / N). Result ends in the returned buffer.
__device__ float2* fft4096(float2* x, float2* y, const float2* __restrict__ tw) {
  for (int ns = 1; ns < N; ns *= 4) {
    const int stride_tw = N / (4 * ns);
    for (int j = threadIdx.x; j < N / 4; j += blockDim.x) {
      const int k = j % ns;
      float2 a0 = x[j];
      float2 a1 = x[j + N / 4];
      float2 a2 = x[j + N / 2];
      float2 a3 = x[j + 3 * N / 4];
      if (ns > 1) {
        a1 = cmul(a1, __ldg(tw + ((1 * k * stride_tw) & (N - 1))));
        a2 = cmul(a2, __ldg(tw + ((2 * k * stride_tw) & (N - 1))));
        a3 = cmul(a3, __ldg(tw + ((3 * k * stride_tw) & (N - 1))));
      }
      // Radix-4 DFT with W4 = -i.
      float2 s02 = make_float2(a0.x + a2.x, a0.y + a2.y);
      float2 d02 = make_float2(a0.x - a2.x, a0.y - a2.y);
      float2 s13 = make_float2(a1.x + a3.x, a1.y + a3.y);
      float2 d13 = make_float2(a1.x - a3.x, a1.y - a3.y);
      const int idx = (j / ns) * ns * 4 + k;
      y[idx] = make_float2(s02.x + s13.x, s02.y + s13.y);
      y[idx + ns] = make_float2(d02.x + d13.y, d02.y - d13.x);      // d02 - i d13
      y[idx + 2 * ns] = make_float2(s02.x - s13.x, s02.y - s13.y);
      y[idx + 3 * ns] = make_float2(d02.x - d13.y, d02.y + d13.x);  // d02 + i d13
    }
    __syncthreads();
    float2* t = x;
    x = y;
    y = t;
  }
  return x;
}

__device__ __forceinline__ int reflect(int i, int n) {
  if (i < 0) i = -i;
  if (i >= n) i = 2 * (n - 1) - i;
  return i;
}

// One CTA per (frame, batch). spec: [B, N/2, frames, 4].
__global__ void __launch_bounds__(NT) stft_cac_kernel(const float* __restrict__ mix, float* __restrict__ spec,
                                                      const float* __restrict__ window,
                                                      const float2* __restrict__ tw, int length, int frames) {
  extern __shared__ __align__(16) float2 sbuf[];
  float2* xa = sbuf;
  float2* xb = sbuf + N;
  const int t = blockIdx.x;
  const int b = blockIdx.y;
  const float* m0 = mix + (long long)b * 2 * length;
  const float* m1 = m0 + length;
  const int base = t * HOP - (HOP / 2 * 3);
  for (int n = threadIdx.x; n < N; n += blockDim.x) {
    int src = reflect(base + n, length);
    float w = __ldg(window + n);
    xa[n] = make_float2(w * __ldg(m0 + src), w * __ldg(m1 + src));
  }
  __syncthreads();
  float2* Z = fft4096(xa, xb, tw);
  const float norm = 0.015625f;  // 1/sqrt(4096)
  float* out = spec + (long long)b * (N / 2) * frames * 4;
  for (int k = threadIdx.x; k < N / 2; k += blockDim.x) {
    float2 zk = Z[k];
    float2 zc = Z[(N - k) & (N - 1)];
    // X0 = (Z[k] + conj(Z[N-k])) / 2 ; X1 = (Z[k] - conj(Z[N-k])) / (2i)
    float4 o;
    o.x = 0.5f * (zk.x + zc.x) * norm;
    o.y = 0.5f * (zk.y - zc.y) * norm;
    o.z = 0.5f * (zk.y + zc.y) * norm;
    o.w = -0.5f * (zk.x - zc.x) * norm;
    *reinterpret_cast<float4*>(out + ((long long)k * frames + t) * 4) = o;
  }
}

// One CTA per (frame, source, batch): inverse FFT of both channels, windowed,
// into frames_buf[b, s, c, t, n].
__global__ void __launch_bounds__(NT) istft_frames_kernel(const float* __restrict__ spec,
                                                          const float* __restrict__ fstats,
                                                          const float* __restrict__ window,
                                                          const float2* __restrict__ tw,
                                                          float* __restrict__ frames_buf, int frames,
                                                          int sources) {
  extern __shared__ __align__(16) float2 sbuf[];
  float2* xa = sbuf;
  float2* xb = sbuf + N;
  const int t = blockIdx.x;
  const int s = blockIdx.y;
  const int b = blockIdx.z;
  const float mean = fstats[2 * b], stdv = fstats[2 * b + 1];
  const int C4 = sources * 4;
  const float* sp = spec + (long long)b * (N / 2) * frames * C4 + (long long)t * C4 + s * 4;
  // Build conj(Z) for the inverse transform via the forward FFT:
  // ifft(Z) = conj(fft(conj(Z))) / N, with Z[k] = X0[k] + i X1[k] and
  // X_c[N-k] = conj(X_c[k]). DC imaginary parts and the Nyquist bin are zero.
  for (int k = threadIdx.x; k <= N / 2; k += blockDim.x) {
    float2 x0 = make_float2(0.f, 0.f), x1 = make_float2(0.f, 0.f);
    if (k < N / 2) {
      float4 v = *reinterpret_cast<const float4*>(sp + (long long)k * frames * C4);
      x0 = make_float2(v.x * stdv + mean, v.y * stdv + mean);
      x1 = make_float2(v.z * stdv + mean, v.w * stdv + mean);
      if (k == 0) {
        x0.y = 0.f;
        x1.y = 0.f;
      }
    }
    // Z[k] = x0 + i x1 ; Z[N-k] = conj(x0) + i conj(x1)
    float2 zk = make_float2(x0.x - x1.y, x0.y + x1.x);
    xa[k] = make_float2(zk.x, -zk.y);
    if (k > 0 && k < N / 2) {
      float2 zn = make_float2(x0.x + x1.y, -x0.y + x1.x);
      xa[N - k] = make_float2(zn.x, -zn.y);
    }
  }
  __syncthreads();
  float2* z = fft4096(xa, xb, tw);
  // z holds fft(conj(Z)) = N * conj(x0 + i x1): x0 = Re(z)/N, x1 = -Im(z)/N.
  const float scale = 0.015625f;  // sqrt(N) / N
  float* f0 = frames_buf + (((long long)b * sources + s) * 2 * frames + t) * N;
  float* f1 = f0 + (long long)frames * N;
  for (int n = threadIdx.x; n < N; n += blockDim.x) {
    float w = __ldg(window + n) * scale;
    float2 v = z[n];
    f0[n] = v.x * w;
    f1[n] = -v.y * w;
  }
}

// out[b, s, c, m] = OLA(frames)[m + crop] / env + xt[b, m, s*2+c] * stdt + meant.
__global__ void istft_ola_kernel(const float* __restrict__ frames_buf, const float* __restrict__ xt,
                                 long long xt_sb, const float* __restrict__ tstats,
                                 const float* __restrict__ window, float* __restrict__ out, int batch,
                                 int sources, int length, int frames) {
  const long long total = (long long)batch * sources * 2 * length;
  // Frame j of the padded istft holds spectrum frame t = j - 2; the padded
  // frame count is frames + 4 and the output sample m sits at OLA position
  // m + 3*HOP/2 (the _ispec crop) + N/2 (the centre crop).
  const int off = HOP / 2 * 3 + N / 2;
  const int jmax = frames + 4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int m = (int)(i % length);
    const long long rc = i / length;  // (b, s, c)
    const int c = (int)(rc % 2);
    const int s = (int)((rc / 2) % sources);
    const int b = (int)(rc / (2 * sources));
    const int n = m + off;
    int j0 = (n - (N - 1) + HOP - 1) / HOP;
    if (n - (N - 1) <= 0) j0 = 0;
    int j1 = n / HOP;
    if (j1 > jmax - 1) j1 = jmax - 1;
    float acc = 0.f, env = 0.f;
    const float* fb = frames_buf + (rc * frames) * (long long)N;
    for (int j = j0; j <= j1; ++j) {
      const int p = n - j * HOP;
      const float w = __ldg(window + p);
      env += w * w;
      const int t = j - 2;
      if (t >= 0 && t < frames) acc += fb[(long long)t * N + p];
    }
    float v = env > 1e-11f ? acc / env : 0.f;
    const float meant = tstats[2 * b], stdt = tstats[2 * b + 1];
    v += xt[(long long)b * xt_sb + (long long)m * (sources * 2) + s * 2 + c] * stdt + meant;
    out[i] = v;
  }
}

}  // namespace

// exp(-2 pi i m / 4096), computed in double and rounded once to float by the
// build step that generates twiddle4096.inc. Static module data: no runtime
// initialisation and no allocation.
__device__ const float2 kTwiddle4096[N] = {
#include "twiddle4096.inc"
};

namespace {
const float2* current_twiddles() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, kTwiddle4096) != cudaSuccess) return nullptr;
  return reinterpret_cast<const float2*>(p);
}
}  // namespace

extern "C" int unblend_stft_cac(const float* mix, float* spec, const float* window, int batch, int length,
                                int nfft, void* stream) {
  UB_REQUIRE(mix && spec && window && batch > 0 && nfft == N);
  UB_REQUIRE(length > HOP / 2 * 3 + HOP);  // reflect padding needs length > pad
  const float2* tw = current_twiddles();
  UB_REQUIRE(tw);
  const int frames = (length + HOP - 1) / HOP;
  const size_t smem = 2 * N * sizeof(float2);
  cudaFuncSetAttribute(stft_cac_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  stft_cac_kernel<<<dim3(frames, batch), NT, smem, ub::as_stream(stream)>>>(mix, spec, window, tw, length,
                                                                           frames);
  UB_CHECK_LAUNCH();
  return 0;
}

// ---------------------------------------------------------------------------
// BS-RoFormer STFT / iSTFT (unblend/roformer.py:1312-1379): torch.stft and
// torch.istft with center=True (reflect pad n/2), not normalized, Hann window
// of length n, any hop; n = 2048 or 4096.
namespace {

// Complex FFT of n = 2^k points (n <= 4096) in shared memory: radix-4
// Stockham stages, then one radix-2 stage when k is odd. tw = exp(-2 pi i m / 4096).
__device__ float2* fft_pow2(float2* x, float2* y, const float2* __restrict__ tw, int n) {
  int ns = 1;
  for (; ns * 4 <= n; ns *= 4) {
    const int tws = 4096 / (4 * ns);
    for (int j = threadIdx.x; j < n / 4; j += blockDim.x) {
      const int k = j % ns;
      float2 a0 = x[j];
      float2 a1 = x[j + n / 4];
      float2 a2 = x[j + n / 2];
      float2 a3 = x[j + 3 * n / 4];
      if (ns > 1) {
        a1 = cmul(a1, __ldg(tw + ((1 * k * tws) & 4095)));
        a2 = cmul(a2, __ldg(tw + ((2 * k * tws) & 4095)));
        a3 = cmul(a3, __ldg(tw + ((3 * k * tws) & 4095)));
      }
      float2 s02 = make_float2(a0.x + a2.x, a0.y + a2.y);
      float2 d02 = make_float2(a0.x - a2.x, a0.y - a2.y);
      float2 s13 = make_float2(a1.x + a3.x, a1.y + a3.y);
      float2 d13 = make_float2(a1.x - a3.x, a1.y - a3.y);
      const int idx = (j / ns) * ns * 4 + k;
      y[idx] = make_float2(s02.x + s13.x, s02.y + s13.y);
      y[idx + ns] = make_float2(d02.x + d13.y, d02.y - d13.x);
      y[idx + 2 * ns] = make_float2(s02.x - s13.x, s02.y - s13.y);
      y[idx + 3 * ns] = make_float2(d02.x - d13.y, d02.y + d13.x);
    }
    __syncthreads();
    float2* t = x;
    x = y;
    y = t;
  }
  if (ns < n) {
    const int tws = 4096 / (2 * ns);
    for (int j = threadIdx.x; j < n / 2; j += blockDim.x) {
      const int k = j % ns;
      const float2 a0 = x[j];
      const float2 a1 = cmul(x[j + n / 2], __ldg(tw + ((k * tws) & 4095)));
      const int idx = (j / ns) * ns * 2 + k;
      y[idx] = make_float2(a0.x + a1.x, a0.y + a1.y);
      y[idx + ns] = make_float2(a0.x - a1.x, a0.y - a1.y);
    }
    __syncthreads();
    float2* t = x;
    x = y;
    y = t;
  }
  return x;
}

// One CTA per (frame, batch): out[b, t, k, c, re/im] for k in [0, n/2].
__global__ void __launch_bounds__(NT) stft_frames_kernel(const float* __restrict__ mix, float* __restrict__ out,
                                                         const float* __restrict__ window,
                                                         const float2* __restrict__ tw, int length, int frames,
                                                         int n, int hop) {
  extern __shared__ __align__(16) float2 sbuf[];
  float2* xa = sbuf;
  float2* xb = sbuf + n;
  const int t = blockIdx.x, b = blockIdx.y;
  const float* m0 = mix + (long long)b * 2 * length;
  const float* m1 = m0 + length;
  const int base = t * hop - n / 2;
  for (int q = threadIdx.x; q < n; q += blockDim.x) {
    const int src = reflect(base + q, length);
    const float w = __ldg(window + q);
    xa[q] = make_float2(w * __ldg(m0 + src), w * __ldg(m1 + src));
  }
  __syncthreads();
  float2* Z = fft_pow2(xa, xb, tw, n);
  const int bins = n / 2 + 1;
  float* o = out + ((long long)b * frames + t) * bins * 4;
  for (int k = threadIdx.x; k < bins; k += blockDim.x) {
    const float2 zk = Z[k & (n - 1)];
    const float2 zc = Z[(n - k) & (n - 1)];
    float4 v;
    v.x = 0.5f * (zk.x + zc.x);
    v.y = 0.5f * (zk.y - zc.y);
    v.z = 0.5f * (zk.y + zc.y);
    v.w = -0.5f * (zk.x - zc.x);
    *reinterpret_cast<float4*>(o + (long long)k * 4) = v;
  }
}

// One CTA per (frame, stem, batch): X_c = stft * mask (complex), DC zeroed,
// inverse real FFT of both channels, times the window, into
// frames_buf[b, s, c, t, q].
__global__ void __launch_bounds__(NT) istft_mask_frames_kernel(const float* __restrict__ stft,
                                                               const float* __restrict__ mask, long long mask_ss,
                                                               const float* __restrict__ window,
                                                               const float2* __restrict__ tw,
                                                               float* __restrict__ frames_buf, int frames,
                                                               int stems, int n, int zero_dc) {
  extern __shared__ __align__(16) float2 sbuf[];
  float2* xa = sbuf;
  float2* xb = sbuf + n;
  const int t = blockIdx.x, s = blockIdx.y, b = blockIdx.z;
  const int bins = n / 2 + 1;
  const float* sp = stft + ((long long)b * frames + t) * bins * 4;
  const float* mp = mask + (long long)s * mask_ss + ((long long)b * frames + t) * bins * 4;
  for (int k = threadIdx.x; k < bins; k += blockDim.x) {
    const float4 a = *reinterpret_cast<const float4*>(sp + (long long)k * 4);
    const float4 m = *reinterpret_cast<const float4*>(mp + (long long)k * 4);
    float2 x0 = make_float2(a.x * m.x - a.y * m.y, a.x * m.y + a.y * m.x);
    float2 x1 = make_float2(a.z * m.z - a.w * m.w, a.z * m.w + a.w * m.z);
    if (k == 0 && zero_dc) x0 = x1 = make_float2(0.f, 0.f);
    if (k == 0 || k == n / 2) {  // a real inverse transform ignores these imaginary parts
      x0.y = 0.f;
      x1.y = 0.f;
    }
    const float2 zk = make_float2(x0.x - x1.y, x0.y + x1.x);  // Z[k] = x0 + i x1
    xa[k] = make_float2(zk.x, -zk.y);
    if (k > 0 && k < n / 2) {
      const float2 zn = make_float2(x0.x + x1.y, -x0.y + x1.x);  // Z[n-k] = conj(x0) + i conj(x1)
      xa[n - k] = make_float2(zn.x, -zn.y);
    }
  }
  __syncthreads();
  float2* z = fft_pow2(xa, xb, tw, n);
  const float inv_n = 1.0f / (float)n;
  float* f0 = frames_buf + (((long long)b * stems + s) * 2 * frames + t) * n;
  float* f1 = f0 + (long long)frames * n;
  for (int q = threadIdx.x; q < n; q += blockDim.x) {
    const float w = __ldg(window + q) * inv_n;
    const float2 v = z[q];
    f0[q] = v.x * w;
    f1[q] = -v.y * w;
  }
}

// out[b, s, c, m] = OLA(frames)[m + n/2] / window-square envelope; with
// `complement`, stem `stems` is mix - stem 0.
__global__ void istft_ola_kernel_any(const float* __restrict__ frames_buf, const float* __restrict__ window,
                                     const float* __restrict__ mix, float* __restrict__ out, int batch, int stems,
                                     int out_stems, int length, int frames, int n, int hop) {
  const long long total = (long long)batch * stems * 2 * length;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int m = (int)(i % length);
    const long long rc = i / length;  // (b, s, c)
    const int c = (int)(rc % 2);
    const int s = (int)((rc / 2) % stems);
    const int b = (int)(rc / (2 * stems));
    const int pos = m + n / 2;
    int j0 = pos - (n - 1) > 0 ? (pos - (n - 1) + hop - 1) / hop : 0;
    int j1 = pos / hop;
    if (j1 > frames - 1) j1 = frames - 1;
    const float* fb = frames_buf + rc * frames * (long long)n;
    float acc = 0.f, env = 0.f;
    for (int j = j0; j <= j1; ++j) {
      const int p = pos - j * hop;
      const float w = __ldg(window + p);
      env += w * w;
      acc += fb[(long long)j * n + p];
    }
    const float v = env > 1e-11f ? acc / env : 0.f;
    out[(((long long)b * out_stems + s) * 2 + c) * length + m] = v;
    if (out_stems > stems)
      out[(((long long)b * out_stems + stems) * 2 + c) * length + m] =
          __ldg(mix + ((long long)b * 2 + c) * length + m) - v;
  }
}

}  // namespace

extern "C" int unblend_stft_frames(const float* mix, float* out, const float* window, int batch, int length,
                                   int nfft, int hop, void* stream) {
  UB_REQUIRE(mix && out && window && batch > 0 && batch < 65536 && (nfft == 2048 || nfft == 4096) && hop > 0);
  UB_REQUIRE(length > nfft / 2);
  const float2* tw = current_twiddles();
  UB_REQUIRE(tw);
  const int frames = 1 + length / hop;
  const size_t smem = 2 * (size_t)nfft * sizeof(float2);
  cudaFuncSetAttribute(stft_frames_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  stft_frames_kernel<<<dim3(frames, batch), NT, smem, ub::as_stream(stream)>>>(mix, out, window, tw, length, frames,
                                                                              nfft, hop);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_istft_masked(const float* stft, const float* mask, long long mask_ss, const float* window,
                                    const float* mix, float* frames_buf, float* out, int batch, int stems,
                                    int complement, int length, int nfft, int hop, int zero_dc, void* stream) {
  UB_REQUIRE(stft && mask && window && frames_buf && out && batch > 0 && stems > 0 && length > 0 && hop > 0);
  UB_REQUIRE((nfft == 2048 || nfft == 4096) && batch < 65536 && stems < 65536);
  UB_REQUIRE(!complement || (stems == 1 && mix));
  const float2* tw = current_twiddles();
  UB_REQUIRE(tw);
  const int frames = 1 + length / hop;
  const size_t smem = 2 * (size_t)nfft * sizeof(float2);
  cudaFuncSetAttribute(istft_mask_frames_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  istft_mask_frames_kernel<<<dim3(frames, stems, batch), NT, smem, ub::as_stream(stream)>>>(
      stft, mask, mask_ss, window, tw, frames_buf, frames, stems, nfft, zero_dc);
  UB_CHECK_LAUNCH();
  const long long total = (long long)batch * stems * 2 * length;
  istft_ola_kernel_any<<<ub::grid_1d(total, 256), 256, 0, ub::as_stream(stream)>>>(
      frames_buf, window, mix, out, batch, stems, stems + (complement ? 1 : 0), length, frames, nfft, hop);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_istft_output(const float* spec, const float* xt, long long xt_sb, const float* fstats,
                                    const float* tstats, const float* window, float* frames_buf, float* out,
                                    int batch, int sources, int length, int nfft, void* stream) {
  UB_REQUIRE(spec && xt && fstats && tstats && window && frames_buf && out);
  UB_REQUIRE(batch > 0 && sources > 0 && length > 0 && nfft == N && sources < 65536);
  const float2* tw = current_twiddles();
  UB_REQUIRE(tw);
  const int frames = (length + HOP - 1) / HOP;
  const size_t smem = 2 * N * sizeof(float2);
  cudaFuncSetAttribute(istft_frames_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  istft_frames_kernel<<<dim3(frames, sources, batch), NT, smem, ub::as_stream(stream)>>>(
      spec, fstats, window, tw, frames_buf, frames, sources);
  UB_CHECK_LAUNCH();
  const long long total = (long long)batch * sources * 2 * length;
  istft_ola_kernel<<<ub::grid_1d(total, 256), 256, 0, ub::as_stream(stream)>>>(
      frames_buf, xt, xt_sb, tstats, window, out, batch, sources, length, frames);
  UB_CHECK_LAUNCH();
  return 0;
}
