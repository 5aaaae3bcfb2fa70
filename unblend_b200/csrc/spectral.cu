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
constexpr int NT = 256;  // one thread per 16 points of a 4096-point transform

__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}

// Twiddles exp(-2 pi i m / 4096) from the first quadrant kept in shared
// memory (tq[r] for r < 1024): m = 1024 q + r is tq[r] times (-i)^q. The
// full table in global memory was re-read from L2 by every stage of every
// transform (its L1 share is small next to the FFT buffers).
constexpr int TQ = 1024;

__device__ __forceinline__ void load_quarter_twiddles(float2* tq, const float2* __restrict__ tw) {
  for (int i = threadIdx.x; i < TQ; i += blockDim.x) tq[i] = __ldg(tw + i);
}

__device__ __forceinline__ float2 twq(const float2* tq, int m) {
  const float2 v = tq[m & (TQ - 1)];
  switch ((m >> 10) & 3) {
    case 0: return v;
    case 1: return make_float2(v.y, -v.x);
    case 2: return make_float2(-v.x, -v.y);
    default: return make_float2(-v.y, v.x);
  }
}

// Forward complex FFT of N = 4096 points in place in shared memory: three
// radix-16 Stockham passes (the autosort formulation, natural order in and
// out). Thread j (256 threads) loads points j + 256 r (r < 16), applies the
// pass twiddles, runs a 16-point DFT in registers (4 x 4 with the W16
// constants between the halves), and after a barrier stores its 16 outputs
// to (j / Ns) * 16 Ns + j % Ns + q Ns. The buffer is padded by one slot per
// 16 (index i -> i + i/16) so the strided stores of the first passes do not
// pile onto a few banks.
constexpr int FFT_BUF = N + N / 16;

__device__ __forceinline__ int pad16(int i) { return i + (i >> 4); }

__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 csub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }

__device__ __forceinline__ void dft4(float2& x0, float2& x1, float2& x2, float2& x3) {
  const float2 s02 = cadd(x0, x2), d02 = csub(x0, x2), s13 = cadd(x1, x3), d13 = csub(x1, x3);
  x0 = cadd(s02, s13);
  x1 = make_float2(d02.x + d13.y, d02.y - d13.x);  // d02 - i d13
  x2 = csub(s02, s13);
  x3 = make_float2(d02.x - d13.y, d02.y + d13.x);  // d02 + i d13
}

// In-register 16-point DFT of a[r]; on return a[4 q1 + q2] holds output q1 + 4 q2.
__device__ __forceinline__ void dft16(float2 (&a)[16]) {
  constexpr float C1 = 0.92387953251128674f, S1 = 0.38268343236508978f, R2 = 0.70710678118654752f;
#pragma unroll
  for (int n1 = 0; n1 < 4; ++n1) dft4(a[n1], a[n1 + 4], a[n1 + 8], a[n1 + 12]);
  // a[n1 + 4 q1] *= exp(-2 pi i n1 q1 / 16)
  a[5] = cmul(a[5], make_float2(C1, -S1));
  a[9] = cmul(a[9], make_float2(R2, -R2));
  a[13] = cmul(a[13], make_float2(S1, -C1));
  a[6] = cmul(a[6], make_float2(R2, -R2));
  a[10] = make_float2(a[10].y, -a[10].x);
  a[14] = cmul(a[14], make_float2(-R2, -R2));
  a[7] = cmul(a[7], make_float2(S1, -C1));
  a[11] = cmul(a[11], make_float2(-R2, -R2));
  a[15] = cmul(a[15], make_float2(-C1, S1));
#pragma unroll
  for (int q1 = 0; q1 < 4; ++q1) dft4(a[4 * q1], a[4 * q1 + 1], a[4 * q1 + 2], a[4 * q1 + 3]);
}

// buf: FFT_BUF float2 (padded layout, pad16 of the natural index); blockDim.x == 256.
__device__ void fft4096(float2* buf, const float2* tq) {
  const int j = threadIdx.x;
#pragma unroll 1
  for (int ls = 0; ls < 12; ls += 4) {  // Ns = 16^pass = 2^ls
    const int ns = 1 << ls;
    const int k = j & (ns - 1);
    float2 a[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) a[r] = buf[pad16(j + 256 * r)];
    if (ls > 0) {
      const int step = k * (N >> (ls + 4));  // k * N / (16 Ns)
#pragma unroll
      for (int r = 1; r < 16; ++r) a[r] = cmul(a[r], twq(tq, (r * step) & (N - 1)));
    }
    dft16(a);
    __syncthreads();  // every point of this pass is in registers before the buffer is overwritten
    const int idx = ((j >> ls) << (ls + 4)) + k;
#pragma unroll
    for (int q = 0; q < 16; ++q) buf[pad16(idx + q * ns)] = a[4 * (q & 3) + (q >> 2)];
    __syncthreads();
  }
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
  float2* xa = sbuf;  // FFT_BUF, padded layout
  float2* tq = sbuf + FFT_BUF;
  load_quarter_twiddles(tq, tw);
  const int t = blockIdx.x;
  const int b = blockIdx.y;
  const float* m0 = mix + (long long)b * 2 * length;
  const float* m1 = m0 + length;
  const int base = t * HOP - (HOP / 2 * 3);
  // Fully unrolled so that all of a thread's global loads are in flight at once.
#pragma unroll
  for (int i = 0; i < N / NT; ++i) {
    const int n = threadIdx.x + i * NT;
    int src = reflect(base + n, length);
    float w = __ldg(window + n);
    xa[pad16(n)] = make_float2(w * __ldg(m0 + src), w * __ldg(m1 + src));
  }
  __syncthreads();
  fft4096(xa, tq);
  const float2* Z = xa;
  const float norm = 0.015625f;  // 1/sqrt(4096)
  float* out = spec + (long long)b * (N / 2) * frames * 4;
  for (int k = threadIdx.x; k < N / 2; k += blockDim.x) {
    float2 zk = Z[pad16(k)];
    float2 zc = Z[pad16((N - k) & (N - 1))];
    // X0 = (Z[k] + conj(Z[N-k])) / 2 ; X1 = (Z[k] - conj(Z[N-k])) / (2i)
    float4 o;
    o.x = 0.5f * (zk.x + zc.x) * norm;
    o.y = 0.5f * (zk.y - zc.y) * norm;
    o.z = 0.5f * (zk.y + zc.y) * norm;
    o.w = -0.5f * (zk.x - zc.x) * norm;
    *reinterpret_cast<float4*>(out + ((long long)k * frames + t) * 4) = o;
  }
}

// One CTA per (source, frame, batch): inverse FFT of both channels, windowed,
// into frames_buf[b, s, c, t, n].
__global__ void __launch_bounds__(NT) istft_frames_kernel(const float* __restrict__ spec,
                                                          const float* __restrict__ fstats,
                                                          const float* __restrict__ window,
                                                          const float2* __restrict__ tw,
                                                          float* __restrict__ frames_buf, int frames,
                                                          int sources) {
  extern __shared__ __align__(16) float2 sbuf[];
  float2* xa = sbuf;  // FFT_BUF, padded layout
  float2* tq = sbuf + FFT_BUF;
  load_quarter_twiddles(tq, tw);
  // Sources vary fastest across CTAs: the four sources of a frame read the
  // same 64-byte runs of the spectrogram at about the same time.
  const int s = blockIdx.x % sources;
  const int t = blockIdx.x / sources;
  const int b = blockIdx.y;
  const float mean = fstats[2 * b], stdv = fstats[2 * b + 1];
  const int C4 = sources * 4;
  const float* sp = spec + (long long)b * (N / 2) * frames * C4 + (long long)t * C4 + s * 4;
  // Build conj(Z) for the inverse transform via the forward FFT:
  // ifft(Z) = conj(fft(conj(Z))) / N, with Z[k] = X0[k] + i X1[k] and
  // X_c[N-k] = conj(X_c[k]). DC imaginary parts and the Nyquist bin are zero.
  // The bins of this (frame, source) sit frames*C4 floats apart: load all of
  // a thread's bins first (independent loads in flight together), then
  // scatter them into the FFT buffer.
  float4 bins[N / 2 / NT];
#pragma unroll
  for (int i = 0; i < N / 2 / NT; ++i)
    bins[i] = __ldg(reinterpret_cast<const float4*>(sp + (long long)(threadIdx.x + i * NT) * frames * C4));
#pragma unroll
  for (int i = 0; i <= N / 2 / NT; ++i) {
    const int k = threadIdx.x + i * NT;
    if (i == N / 2 / NT && k != N / 2) break;
    float2 x0 = make_float2(0.f, 0.f), x1 = make_float2(0.f, 0.f);
    if (i < N / 2 / NT) {  // k < N/2; k == N/2 is the Nyquist bin (zero)
      const float4 v = bins[i < N / 2 / NT ? i : 0];
      x0 = make_float2(v.x * stdv + mean, v.y * stdv + mean);
      x1 = make_float2(v.z * stdv + mean, v.w * stdv + mean);
      if (k == 0) {
        x0.y = 0.f;
        x1.y = 0.f;
      }
    }
    // Z[k] = x0 + i x1 ; Z[N-k] = conj(x0) + i conj(x1)
    float2 zk = make_float2(x0.x - x1.y, x0.y + x1.x);
    xa[pad16(k)] = make_float2(zk.x, -zk.y);
    if (k > 0 && k < N / 2) {
      float2 zn = make_float2(x0.x + x1.y, -x0.y + x1.x);
      xa[pad16(N - k)] = make_float2(zn.x, -zn.y);
    }
  }
  __syncthreads();
  fft4096(xa, tq);
  const float2* z = xa;
  // z holds fft(conj(Z)) = N * conj(x0 + i x1): x0 = Re(z)/N, x1 = -Im(z)/N.
  const float scale = 0.015625f;  // sqrt(N) / N
  float* f0 = frames_buf + (((long long)b * sources + s) * 2 * frames + t) * N;
  float* f1 = f0 + (long long)frames * N;
  for (int n = threadIdx.x; n < N; n += blockDim.x) {
    float w = __ldg(window + n) * scale;
    float2 v = z[pad16(n)];
    f0[n] = v.x * w;
    f1[n] = -v.y * w;
  }
}

// out[b, s, c, m] = OLA(frames)[m + crop] / env + xt[b, m, s*2+c] * stdt + meant.
// One CTA per (block of OLA_M samples, batch): the time-branch rows of the
// block (all sources and channels, contiguous in xt) are staged in shared
// memory so that both xt and out are accessed in contiguous runs.
constexpr int OLA_M = 64;
constexpr int OLA_MAXP = 32;  // sources * 2 planes at most

__global__ void __launch_bounds__(256) istft_ola_kernel(const float* __restrict__ frames_buf,
                                                        const float* __restrict__ xt, long long xt_sb,
                                                        const float* __restrict__ tstats,
                                                        const float* __restrict__ window, float* __restrict__ out,
                                                        int sources, int length, int frames) {
  __shared__ float xs[OLA_M * OLA_MAXP];
  const int planes = sources * 2;
  const int b = blockIdx.y;
  const int m0 = blockIdx.x * OLA_M;
  const int nm = min(OLA_M, length - m0);
  const float* xb = xt + (long long)b * xt_sb + (long long)m0 * planes;
  for (int i = threadIdx.x; i < nm * planes; i += blockDim.x) xs[i] = __ldg(xb + i);
  __syncthreads();
  // Frame j of the padded istft holds spectrum frame t = j - 2; the padded
  // frame count is frames + 4 and the output sample m sits at OLA position
  // m + 3*HOP/2 (the _ispec crop) + N/2 (the centre crop).
  const int off = HOP / 2 * 3 + N / 2;
  const int jmax = frames + 4;
  const float meant = tstats[2 * b], stdt = tstats[2 * b + 1];
  for (int i = threadIdx.x; i < planes * OLA_M; i += blockDim.x) {
    const int pl = i / OLA_M, mm = i - pl * OLA_M;
    if (mm >= nm) continue;
    const int m = m0 + mm;
    const int n = m + off;
    int j0 = (n - (N - 1) + HOP - 1) / HOP;
    if (n - (N - 1) <= 0) j0 = 0;
    int j1 = n / HOP;
    if (j1 > jmax - 1) j1 = jmax - 1;
    float acc = 0.f, env = 0.f;
    const float* fb = frames_buf + ((long long)b * planes + pl) * frames * (long long)N;
    for (int j = j0; j <= j1; ++j) {
      const int p = n - j * HOP;
      const float w = __ldg(window + p);
      env += w * w;
      const int t = j - 2;
      if (t >= 0 && t < frames) acc += fb[(long long)t * N + p];
    }
    float v = env > 1e-11f ? acc / env : 0.f;
    v += xs[mm * planes + pl] * stdt + meant;
    out[((long long)b * planes + pl) * length + m] = v;
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
  const size_t smem = (FFT_BUF + TQ) * sizeof(float2);
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
__device__ float2* fft_pow2(float2* x, float2* y, const float2* tq, int n) {
  int ns = 1, ls = 0;  // ns = 2^ls
  for (; ns * 4 <= n; ns *= 4, ls += 2) {
    const int tws = 4096 / (4 * ns);
    for (int j = threadIdx.x; j < n / 4; j += blockDim.x) {
      const int k = j & (ns - 1);
      float2 a0 = x[j];
      float2 a1 = x[j + n / 4];
      float2 a2 = x[j + n / 2];
      float2 a3 = x[j + 3 * n / 4];
      if (ns > 1) {
        a1 = cmul(a1, twq(tq, (1 * k * tws) & 4095));
        a2 = cmul(a2, twq(tq, (2 * k * tws) & 4095));
        a3 = cmul(a3, twq(tq, (3 * k * tws) & 4095));
      }
      float2 s02 = make_float2(a0.x + a2.x, a0.y + a2.y);
      float2 d02 = make_float2(a0.x - a2.x, a0.y - a2.y);
      float2 s13 = make_float2(a1.x + a3.x, a1.y + a3.y);
      float2 d13 = make_float2(a1.x - a3.x, a1.y - a3.y);
      const int idx = ((j >> ls) << (ls + 2)) + k;
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
      const float2 a1 = cmul(x[j + n / 2], twq(tq, (k * tws) & 4095));
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
  float2* tq = sbuf + 2 * n;
  load_quarter_twiddles(tq, tw);
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
  float2* Z = fft_pow2(xa, xb, tq, n);
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
  float2* tq = sbuf + 2 * n;
  load_quarter_twiddles(tq, tw);
  const int t = blockIdx.x, s = blockIdx.y, b = blockIdx.z;
  const int bins = n / 2 + 1;
  const float* sp = stft ? stft + ((long long)b * frames + t) * bins * 4 : nullptr;
  const float* mp = mask + (long long)s * mask_ss + ((long long)b * frames + t) * bins * 4;
  for (int k = threadIdx.x; k < bins; k += blockDim.x) {
    // Without a spectrum the mask itself is inverted (a unit complex factor).
    const float4 a = sp ? *reinterpret_cast<const float4*>(sp + (long long)k * 4) : make_float4(1.f, 0.f, 1.f, 0.f);
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
  float2* z = fft_pow2(xa, xb, tq, n);
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
  const size_t smem = (2 * (size_t)nfft + TQ) * sizeof(float2);
  cudaFuncSetAttribute(stft_frames_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  stft_frames_kernel<<<dim3(frames, batch), NT, smem, ub::as_stream(stream)>>>(mix, out, window, tw, length, frames,
                                                                              nfft, hop);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_istft_masked(const float* stft, const float* mask, long long mask_ss, const float* window,
                                    const float* mix, float* frames_buf, float* out, int batch, int stems,
                                    int complement, int length, int nfft, int hop, int zero_dc, void* stream) {
  UB_REQUIRE(mask && window && frames_buf && out && batch > 0 && stems > 0 && length > 0 && hop > 0);
  UB_REQUIRE((nfft == 2048 || nfft == 4096) && batch < 65536 && stems < 65536);
  UB_REQUIRE(!complement || (stems == 1 && mix));
  const float2* tw = current_twiddles();
  UB_REQUIRE(tw);
  const int frames = 1 + length / hop;
  const size_t smem = (2 * (size_t)nfft + TQ) * sizeof(float2);
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
  UB_REQUIRE(batch > 0 && sources > 0 && length > 0 && nfft == N && 2 * sources <= OLA_MAXP);
  UB_REQUIRE(batch < 65536);
  const float2* tw = current_twiddles();
  UB_REQUIRE(tw);
  const int frames = (length + HOP - 1) / HOP;
  const size_t smem = (FFT_BUF + TQ) * sizeof(float2);
  cudaFuncSetAttribute(istft_frames_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  istft_frames_kernel<<<dim3(frames * sources, batch), NT, smem, ub::as_stream(stream)>>>(
      spec, fstats, window, tw, frames_buf, frames, sources);
  UB_CHECK_LAUNCH();
  istft_ola_kernel<<<dim3((length + OLA_M - 1) / OLA_M, batch), 256, 0, ub::as_stream(stream)>>>(
      frames_buf, xt, xt_sb, tstats, window, out, sources, length, frames);
  UB_CHECK_LAUNCH();
  return 0;
}
