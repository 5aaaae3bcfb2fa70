// Host I/O edges of the separation pipeline on the GPU (fp32): 16-bit PCM
// decode with channel conversion, windowed-sinc resampling, and the clipping
// guards applied before export (unblend/api.py:1080-1112 _read_pcm16_wav,
// unblend/audio.py:14-67 convert_audio_channels / convert_audio,
// unblend/audio.py:70-90 prevent_clip), and the 16-bit PCM export of a stem
// (unblend/api.py:94-148 export_stem). Decoding and encoding on the device move
// 2-byte samples over PCIe instead of 4-byte floats.
#include "common.cuh"

namespace {

// Channel conversion of unblend/audio.py:14-48: same count -> copy; one output
// channel -> mean of the inputs (summed in channel order, then divided);
// one input channel -> replicated; more inputs than outputs -> the first ones.
__device__ __forceinline__ float convert_channel(const float* v, int cin, int cout, int c) {
  if (cin == cout) return v[c];
  if (cout == 1) {
    float s = 0.f;
    for (int i = 0; i < cin; ++i) s += v[i];
    return s / (float)cin;
  }
  if (cin == 1) return v[0];
  return v[c];
}

// src: interleaved int16 [frames, cin]; dst: planar fp32 [cout, frames], x / 32768.
__global__ void pcm16_to_f32_kernel(const short* __restrict__ src, int cin, long long frames, float* __restrict__ dst,
                                    int cout) {
  for (long long f = blockIdx.x * (long long)blockDim.x + threadIdx.x; f < frames;
       f += (long long)gridDim.x * blockDim.x) {
    float v[8];
    for (int i = 0; i < cin; ++i) v[i] = (float)__ldg(src + f * cin + i) / 32768.0f;
    for (int c = 0; c < cout; ++c) dst[(long long)c * frames + f] = convert_channel(v, cin, cout, c);
  }
}

// x: planar fp32 [cin, frames] -> y: planar [cout, frames].
__global__ void convert_channels_kernel(const float* __restrict__ x, int cin, long long frames, float* __restrict__ y,
                                        int cout) {
  for (long long f = blockIdx.x * (long long)blockDim.x + threadIdx.x; f < frames;
       f += (long long)gridDim.x * blockDim.x) {
    float v[8];
    for (int i = 0; i < cin; ++i) v[i] = __ldg(x + (long long)i * frames + f);
    for (int c = 0; c < cout; ++c) y[(long long)c * frames + f] = convert_channel(v, cin, cout, c);
  }
}

// Polyphase windowed-sinc resampling. With the rates reduced by their gcd to
// lin -> lout, output sample k * lout + p of a channel is
//   sum_{m < taps} x[k * lin + m - width] * kern[p, m]   (x zero outside [0, length)),
// kern holding one filter row per output phase. Blocks: (frame block, phase);
// a warp walks consecutive frames of one phase, so the filter row is a
// broadcast read and the strided input reads hit L1.
__global__ void resample_kernel(const float* __restrict__ x, int channels, long long length,
                                const float* __restrict__ kern, int taps, int lin, int lout, int width,
                                float* __restrict__ y, long long out_length) {
  const int p = blockIdx.y;
  const float* kr = kern + (long long)p * taps;
  const long long frames = (out_length - p + lout - 1) / lout;  // frames k with k * lout + p < out_length
  for (long long k = blockIdx.x * (long long)blockDim.x + threadIdx.x; k < frames;
       k += (long long)gridDim.x * blockDim.x) {
    const long long base = k * lin - width;
    for (int c = 0; c < channels; ++c) {
      const float* xc = x + (long long)c * length;
      float acc = 0.f;
      if (base >= 0 && base + taps <= length) {
        for (int m = 0; m < taps; ++m) acc = fmaf(__ldg(xc + base + m), __ldg(kr + m), acc);
      } else {
        for (int m = 0; m < taps; ++m) {
          const long long i = base + m;
          if (i >= 0 && i < length) acc = fmaf(__ldg(xc + i), __ldg(kr + m), acc);
        }
      }
      y[(long long)c * out_length + k * lout + p] = acc;
    }
  }
}

// max |x| as float bits (non-negative floats order like their bit patterns).
__global__ void max_abs_kernel(const float* __restrict__ x, long long n, unsigned* __restrict__ out) {
  float m = 0.f;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(__ldg(x + i)));
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));
}

// mode 1 rescale: x / max(1.01 max|x|, 1); 2 clamp to [-0.99, 0.99]; 3 tanh.
__global__ void prevent_clip_kernel(const float* __restrict__ x, float* __restrict__ y, long long n, int mode,
                                    const unsigned* __restrict__ maxabs_bits) {
  const float s = mode == 1 ? fmaxf(1.01f * __uint_as_float(*maxabs_bits), 1.0f) : 1.f;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float v = __ldg(x + i);
    y[i] = mode == 1 ? v / s : mode == 2 ? fminf(fmaxf(v, -0.99f), 0.99f) : tanhf(v);
  }
}

// Export edge: planar fp32 [channels, frames] -> interleaved int16 [frames,
// channels], the clipping guard above applied first (mode 0 = none), then the
// float -> signed 16-bit conversion of FFmpeg's libswresample that the
// reference's encoder runs for a 16-bit PCM WAV stem: round x * 2^15 to the
// nearest integer (ties to even, as lrintf in the default rounding mode) and
// saturate to [-32768, 32767]. NaN samples are written as 0.
__global__ void encode_pcm16_kernel(const float* __restrict__ x, int channels, long long frames, int mode,
                                    const unsigned* __restrict__ maxabs_bits, short* __restrict__ dst) {
  const float s = mode == 1 ? fmaxf(1.01f * __uint_as_float(*maxabs_bits), 1.0f) : 1.f;
  const long long n = frames * channels;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const long long f = i / channels;
    const int c = (int)(i - f * channels);
    float v = __ldg(x + (long long)c * frames + f);
    if (mode == 1) v = v / s;
    else if (mode == 2) v = fminf(fmaxf(v, -0.99f), 0.99f);
    else if (mode == 3) v = tanhf(v);
    int q = __float2int_rn(v * 32768.f);
    q = isnan(v) ? 0 : min(max(q, -32768), 32767);
    dst[i] = (short)q;
  }
}

}  // namespace

extern "C" int unblend_encode_pcm16(const float* x, int channels, long long frames, int mode,
                                    const unsigned* maxabs_bits, void* dst, void* stream) {
  UB_REQUIRE(x && dst && channels > 0 && channels <= 8 && frames > 0 && mode >= 0 && mode <= 3);
  UB_REQUIRE(mode != 1 || maxabs_bits);
  encode_pcm16_kernel<<<ub::grid_1d(frames * channels, 256), 256, 0, ub::as_stream(stream)>>>(
      x, channels, frames, mode, maxabs_bits, reinterpret_cast<short*>(dst));
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_pcm16_to_f32(const void* src, int cin, long long frames, float* dst, int cout, void* stream) {
  UB_REQUIRE(src && dst && frames > 0 && cin > 0 && cin <= 8 && cout > 0 && cout <= 8);
  UB_REQUIRE(cin == cout || cout == 1 || cin == 1 || cin > cout);
  pcm16_to_f32_kernel<<<ub::grid_1d(frames, 256), 256, 0, ub::as_stream(stream)>>>(
      reinterpret_cast<const short*>(src), cin, frames, dst, cout);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_convert_channels(const float* x, int cin, long long frames, float* y, int cout, void* stream) {
  UB_REQUIRE(x && y && frames > 0 && cin > 0 && cin <= 8 && cout > 0 && cout <= 8);
  UB_REQUIRE(cin == cout || cout == 1 || cin == 1 || cin > cout);
  convert_channels_kernel<<<ub::grid_1d(frames, 256), 256, 0, ub::as_stream(stream)>>>(x, cin, frames, y, cout);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_resample(const float* x, int channels, long long length, const float* kern, int taps, int lin,
                                int lout, int width, float* y, long long out_length, void* stream) {
  UB_REQUIRE(x && kern && y && channels > 0 && length > 0 && taps > 0 && lin > 0 && lout > 0 && width >= 0);
  UB_REQUIRE(out_length > 0 && lout < 65536);
  const long long frames = (out_length + lout - 1) / lout;
  dim3 grid((unsigned)((frames + 255) / 256 < 4096 ? (frames + 255) / 256 : 4096), (unsigned)lout);
  resample_kernel<<<grid, 256, 0, ub::as_stream(stream)>>>(x, channels, length, kern, taps, lin, lout, width, y,
                                                           out_length);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_max_abs(const float* x, long long n, unsigned* out_bits, void* stream) {
  UB_REQUIRE(x && out_bits && n > 0);
  max_abs_kernel<<<ub::grid_1d(n, 256), 256, 0, ub::as_stream(stream)>>>(x, n, out_bits);
  UB_CHECK_LAUNCH();
  return 0;
}

extern "C" int unblend_prevent_clip(const float* x, float* y, long long n, int mode, const unsigned* maxabs_bits,
                                    void* stream) {
  UB_REQUIRE(x && y && n > 0 && mode >= 1 && mode <= 3 && (mode != 1 || maxabs_bits));
  prevent_clip_kernel<<<ub::grid_1d(n, 256), 256, 0, ub::as_stream(stream)>>>(x, y, n, mode, maxabs_bits);
  UB_CHECK_LAUNCH();
  return 0;
}
