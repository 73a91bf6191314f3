// logmel.cu -- the Whisper log-mel front end on the GPU: what the reference runs through
// preprocessor.onnx (rust/npu-engine/src/asr/whisper.rs:686-705), an export of the Whisper
// feature extractor: 480,000 samples -> input_features [80][3000].
//
//   frame f (f < 3000) = samples 160 f - 200 .. 160 f + 199 of the clip reflect-padded by 200,
//   times the periodic Hann window; power spectrum of its 400-point DFT (bins 0..200); 80 Slaney
//   mel filters; log10(max(mel, 1e-10)); clamp below at the clip's maximum - 8; (x + 4) / 4.
//
// Kernel 1 (one CTA per clip and 32 frames): the 5,360 samples the frames cover are staged in
// shared memory with the window and a 400-entry cos / sin table; each thread accumulates the
// DFT of 4 frames x 7 bins in f32 registers (the table index k n mod 400 advances by k per
// sample, so no integer multiply or modulo in the loop), writes the powers to shared memory,
// then the mel sums over each filter's nonzero bins, log10, and the block's maximum folded into
// the clip's with an integer atomicMax on the order-preserving encoding of the float.
// Kernel 2: the clamp and scale, elementwise.  The DFT is direct: 201 x 400 multiply-adds per
// frame per component, ~0.5 G per clip, a few tens of microseconds on 148 SMs -- small next to
// the encoder, and free of an FFT's twiddle recurrences.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <string>
#include <vector>

#include "../../include/xdna_b200.h"

namespace xdna {
void set_last_error_message(const std::string &m);
}
using xdna::set_last_error_message;

struct XdnaDevice;
extern "C" int xdna_device_ordinal(const XdnaDevice *dev);

namespace logmel {

constexpr int kFft = 400, kHop = 160, kBins = 201, kMels = 80, kSamples = 480000, kFrames = 3000;
constexpr int kFramesPerCta = 32, kSpan = (kFramesPerCta - 1) * kHop + kFft;   // 5,360 samples
constexpr int kThreads = 256, kBinGroups = 32, kBinsPerThread = 7;              // 32 x 7 = 224 >= 201

struct Tables {
    float cs[kFft], sn[kFft];         // cos / sin(2 pi m / 400)
    float win[kFft];                  // periodic Hann
    float filt[kMels][kBins];         // Slaney filters, mel-major
    int lo[kMels], hi[kMels];         // nonzero bin range [lo, hi) of each filter
};

__device__ __forceinline__ unsigned ordered(float f) {
    const unsigned u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float unordered(unsigned u) {
    return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}

__global__ void __launch_bounds__(kThreads) spectrum_kernel(const float *__restrict__ wav, const Tables *__restrict__ tab,
                                                            float *__restrict__ out, unsigned *__restrict__ clip_max) {
    // the staged samples are dead once the DFT is done: the powers reuse their space
    constexpr int kPwStride = kBins + 3;
    __shared__ float buf[kFramesPerCta * kPwStride > kSpan ? kFramesPerCta * kPwStride : kSpan];
    __shared__ float cs[kFft], sn[kFft], win[kFft];
    float *xs = buf;
    float(*pw)[kPwStride] = reinterpret_cast<float(*)[kPwStride]>(buf);
    __shared__ unsigned bmax;
    const int clip = blockIdx.y, f0 = blockIdx.x * kFramesPerCta, tid = threadIdx.x;
    const float *x = wav + (size_t)clip * kSamples;
    for (int i = tid; i < kSpan; i += kThreads) {
        int s = f0 * kHop - kFft / 2 + i;                  // reflect padding (no edge repeat)
        s = s < 0 ? -s : s;
        s = s >= kSamples ? 2 * (kSamples - 1) - s : s;
        xs[i] = x[s];
    }
    for (int i = tid; i < kFft; i += kThreads) {
        cs[i] = tab->cs[i];
        sn[i] = tab->sn[i];
        win[i] = tab->win[i];
    }
    if (tid == 0) bmax = 0u;
    __syncthreads();
    // thread (fg, bg): frames 4 fg .. 4 fg + 3, bins bg + 32 j
    const int fg = tid / kBinGroups, bg = tid % kBinGroups;
    float re[4][kBinsPerThread], im[4][kBinsPerThread];
#pragma unroll
    for (int a = 0; a < 4; a++)
#pragma unroll
        for (int j = 0; j < kBinsPerThread; j++) re[a][j] = im[a][j] = 0.0f;
    int idx[kBinsPerThread];
#pragma unroll
    for (int j = 0; j < kBinsPerThread; j++) idx[j] = 0;
    const float *xf = xs + 4 * fg * kHop;
    for (int n = 0; n < kFft; n++) {
        const float w = win[n];
        float v[4];
#pragma unroll
        for (int a = 0; a < 4; a++) v[a] = w * xf[a * kHop + n];
#pragma unroll
        for (int j = 0; j < kBinsPerThread; j++) {
            const float c = cs[idx[j]], s = sn[idx[j]];
#pragma unroll
            for (int a = 0; a < 4; a++) {
                re[a][j] = fmaf(v[a], c, re[a][j]);
                im[a][j] = fmaf(v[a], s, im[a][j]);
            }
            idx[j] += bg + kBinGroups * j;
            idx[j] -= idx[j] >= kFft ? kFft : 0;           // k < 400, so one subtraction suffices
        }
    }
    __syncthreads();                                        // every thread is done with xs
#pragma unroll
    for (int j = 0; j < kBinsPerThread; j++) {
        const int k = bg + kBinGroups * j;
        if (k < kBins)
#pragma unroll
            for (int a = 0; a < 4; a++) pw[4 * fg + a][k] = re[a][j] * re[a][j] + im[a][j] * im[a][j];
    }
    __syncthreads();
    // mel + log10: 80 mels x 32 frames, consecutive threads on consecutive frames
    float m_local = -INFINITY;
    for (int o = tid; o < kMels * kFramesPerCta; o += kThreads) {
        const int mel = o / kFramesPerCta, fl = o % kFramesPerCta, f = f0 + fl;
        if (f >= kFrames) continue;
        float acc = 0.0f;
        for (int k = tab->lo[mel]; k < tab->hi[mel]; k++) acc = fmaf(tab->filt[mel][k], pw[fl][k], acc);
        const float lg = log10f(fmaxf(acc, 1e-10f));
        out[((size_t)clip * kMels + mel) * kFrames + f] = lg;
        m_local = fmaxf(m_local, lg);
    }
    const unsigned wm = __reduce_max_sync(0xffffffffu, ordered(m_local));
    if ((tid & 31) == 0) atomicMax(&bmax, wm);
    __syncthreads();
    if (tid == 0) atomicMax(clip_max + clip, bmax);
}

// input_features = (max(x, clip max - 8) + 4) / 4
__global__ void normalize_kernel(float *__restrict__ out, const unsigned *__restrict__ clip_max, int B) {
    const size_t n = (size_t)B * kMels * kFrames;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float lo = unordered(clip_max[i / (kMels * kFrames)]) - 8.0f;
        out[i] = (fmaxf(out[i], lo) + 4.0f) / 4.0f;
    }
}

}  // namespace logmel

struct XdnaLogMel {
    int ordinal = 0;
    logmel::Tables *tab = nullptr;   // device
    unsigned *clip_max = nullptr;    // device, [cap]
    int cap = 0;
    float *wav = nullptr, *mel = nullptr;   // staging for the host form (one clip)
};

namespace {

bool ck(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return true;
    set_last_error_message(std::string(what) + ": " + cudaGetErrorString(e));
    return false;
}

// Slaney mel scale (the Auditory Toolbox's): linear below 1 kHz, logarithmic above
double hz_to_mel(double f) { return f >= 1000.0 ? 15.0 + std::log(f / 1000.0) * (27.0 / std::log(6.4)) : 3.0 * f / 200.0; }
double mel_to_hz(double m) { return m >= 15.0 ? 1000.0 * std::exp((m - 15.0) * (std::log(6.4) / 27.0)) : 200.0 * m / 3.0; }

void build_tables(logmel::Tables &t) {
    using namespace logmel;
    const double pi = 3.14159265358979323846;
    for (int m = 0; m < kFft; m++) {
        t.cs[m] = (float)std::cos(2.0 * pi * m / kFft);
        t.sn[m] = (float)std::sin(2.0 * pi * m / kFft);
        t.win[m] = (float)(0.5 - 0.5 * std::cos(2.0 * pi * m / kFft));
    }
    // centre frequencies: kMels + 2 points evenly spaced in mel over 0 .. 8000 Hz
    double fc[kMels + 2];
    const double m0 = hz_to_mel(0.0), m1 = hz_to_mel(8000.0);
    for (int i = 0; i < kMels + 2; i++) fc[i] = mel_to_hz(m0 + (m1 - m0) * i / (kMels + 1));
    for (int m = 0; m < kMels; m++) {
        const double norm = 2.0 / (fc[m + 2] - fc[m]);
        t.lo[m] = kBins;
        t.hi[m] = 0;
        for (int k = 0; k < kBins; k++) {
            const double f = 8000.0 * k / (kBins - 1);
            const double down = (f - fc[m]) / (fc[m + 1] - fc[m]), up = (fc[m + 2] - f) / (fc[m + 2] - fc[m + 1]);
            const double v = std::max(0.0, std::min(down, up)) * norm;
            t.filt[m][k] = (float)v;
            if (v > 0.0) {
                t.lo[m] = std::min(t.lo[m], k);
                t.hi[m] = k + 1;
            }
        }
        if (t.hi[m] == 0) t.lo[m] = 0;
    }
}

}  // namespace

extern "C" {

XdnaLogMel *xdna_log_mel_create(XdnaDevice *dev) {
    if (!dev) { set_last_error_message("xdna_log_mel_create: null device"); return nullptr; }
    auto *h = new XdnaLogMel();
    h->ordinal = xdna_device_ordinal(dev);
    std::vector<logmel::Tables> t(1);
    build_tables(t[0]);
    if (!ck(cudaSetDevice(h->ordinal), "xdna_log_mel_create") ||
        !ck(cudaMalloc(&h->tab, sizeof(logmel::Tables)), "xdna_log_mel_create") ||
        !ck(cudaMemcpy(h->tab, t.data(), sizeof(logmel::Tables), cudaMemcpyHostToDevice), "xdna_log_mel_create")) {
        xdna_log_mel_free(h);
        return nullptr;
    }
    return h;
}

void xdna_log_mel_free(XdnaLogMel *h) {
    if (!h) return;
    cudaSetDevice(h->ordinal);
    cudaFree(h->tab);
    cudaFree(h->clip_max);
    cudaFree(h->wav);
    cudaFree(h->mel);
    delete h;
}

int xdna_log_mel_device(XdnaLogMel *h, const float *wav_dev, int B, float *mel_dev, void *stream) {
    using namespace logmel;
    if (!h || !wav_dev || !mel_dev || B < 1 || B > 65535) {
        set_last_error_message("xdna_log_mel_device: null pointer or B outside 1..65535");
        return -1;
    }
    if (!ck(cudaSetDevice(h->ordinal), "xdna_log_mel_device")) return -1;
    if (B > h->cap) {
        // grows between calls only; a call in flight on another stream keeps its own size
        if (!ck(cudaDeviceSynchronize(), "xdna_log_mel_device")) return -1;
        cudaFree(h->clip_max);
        h->clip_max = nullptr;
        h->cap = 0;
        if (!ck(cudaMalloc(&h->clip_max, sizeof(unsigned) * B), "xdna_log_mel_device")) return -1;
        h->cap = B;
    }
    auto st = static_cast<cudaStream_t>(stream);
    if (!ck(cudaMemsetAsync(h->clip_max, 0, sizeof(unsigned) * B, st), "xdna_log_mel_device")) return -1;
    spectrum_kernel<<<dim3((kFrames + kFramesPerCta - 1) / kFramesPerCta, B), kThreads, 0, st>>>(wav_dev, h->tab, mel_dev,
                                                                                               h->clip_max);
    normalize_kernel<<<148 * 8, 256, 0, st>>>(mel_dev, h->clip_max, B);
    return ck(cudaGetLastError(), "xdna_log_mel_device") ? 0 : -1;
}

int xdna_log_mel(XdnaLogMel *h, const int16_t *pcm, size_t n, float *mel) {
    using namespace logmel;
    if (!h || (!pcm && n) || !mel) { set_last_error_message("xdna_log_mel: null pointer"); return -1; }
    std::vector<float> wav(kSamples, 0.0f);
    const size_t m = n < (size_t)kSamples ? n : (size_t)kSamples;
    for (size_t i = 0; i < m; i++) wav[i] = (float)pcm[i] / 32768.0f;
    if (!ck(cudaSetDevice(h->ordinal), "xdna_log_mel")) return -1;
    if (!h->wav && (!ck(cudaMalloc(&h->wav, sizeof(float) * kSamples), "xdna_log_mel") ||
                    !ck(cudaMalloc(&h->mel, sizeof(float) * kMels * kFrames), "xdna_log_mel")))
        return -1;
    if (!ck(cudaMemcpy(h->wav, wav.data(), sizeof(float) * kSamples, cudaMemcpyHostToDevice), "xdna_log_mel")) return -1;
    if (xdna_log_mel_device(h, h->wav, 1, h->mel, nullptr) != 0) return -1;
    return ck(cudaMemcpy(mel, h->mel, sizeof(float) * kMels * kFrames, cudaMemcpyDeviceToHost), "xdna_log_mel") ? 0 : -1;
}

}  // extern "C"
