// ASR front-end glue on the device: the log-mel spectrogram of a 16 kHz
// waveform and the assembly of the decoder's input rows from prompt tokens
// and audio embeddings.
//
// b2_log_mel restates MelExtractor.__call__ (examples/qwen3_asr/mel.py:52-67 of
// suharvest/rknn-matmul-parallel) and its _stft_numpy (:6-27):
//   * reflect padding by n_fft / 2 = 200 samples on both sides (center=True),
//   * periodic Hann window w[k] = 0.5 - 0.5 cos(2 pi k / 400), k < 400,
//   * frames every 160 samples, |rfft_400|^2 -> 201 bins,
//   * mel = filters^T . power (filters [201][128], the caller's mel_filters),
//   * log10(max(mel, 1e-10)), clamped below at (max over ALL frames) - 8,
//     then (x + 4) / 4,
//   * the last frame dropped: T = n / 160 output frames of the n / 160 + 1
//     computed ones (the clamp's maximum still sees the dropped frame).
// The DFT runs in FP32 against an FP32 twiddle table (cos and sin of
// 2 pi j / 400, each CTA computing it in double and rounding once); the
// reference's numpy FFT differs by rounding only.
//
// b2_build_embed restates the row assembly of build_embed
// (examples/qwen3_asr/engine.py:255-314): [prefix token rows | audio rows |
// suffix token rows], token rows gathered from the decoder's FP32 embedding
// table.  The token ids themselves come from the caller's tokenizer.
#include "b2_common.cuh"

namespace {

constexpr int kFFT = 400;
constexpr int kHop = 160;
constexpr int kBins = kFFT / 2 + 1;  // 201
constexpr int kMel = 128;
constexpr int kFrames = 8;           // STFT frames per CTA
constexpr int kThreads = 256;
constexpr int kSpan = (kFrames - 1) * kHop + kFFT;  // padded samples a CTA reads
constexpr int kMelWork = 256;        // bytes before the log-mel rows in the workspace (the maximum)

__device__ __forceinline__ float ordered_max_decode(unsigned u) {
    return __uint_as_float((u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u);
}

// One CTA: kFrames consecutive STFT frames -> log10 mel values in
// work[frame][128], and the CTA's maximum folded into *gmax (orderable key).
__global__ void __launch_bounds__(kThreads) log_mel_frames(const float* __restrict__ audio, int n, int n_frames,
                                                          const float* __restrict__ filters, float* __restrict__ work,
                                                          unsigned* __restrict__ gmax) {
    __shared__ float xs[kSpan];                  // padded samples
    __shared__ float xw[kFrames][kFFT];          // windowed frames
    __shared__ float2 tw[kFFT];                  // (cos, sin) of 2 pi j / 400
    __shared__ float win[kFFT];
    __shared__ float pw[kFrames][kBins + 3];     // power spectrum
    __shared__ unsigned red[kThreads / 32];
    const int f0 = blockIdx.x * kFrames;
    for (int j = threadIdx.x; j < kFFT; j += kThreads) {
        double sn, cs;
        sincospi(2.0 * j / kFFT, &sn, &cs);
        tw[j] = make_float2((float)cs, (float)sn);
        win[j] = (float)(0.5 - 0.5 * cs);  // periodic Hann (np.hanning(401)[:400])
    }
    // padded sample p (0 <= p < n + 400) is audio[p - 200] with reflection
    // at both ends (numpy 'reflect': the edge sample is not repeated)
    for (int i = threadIdx.x; i < kSpan; i += kThreads) {
        const int p = f0 * kHop + i;
        float v = 0.f;
        if (p < n + kFFT) {
            int a = p - kFFT / 2;
            if (a < 0) a = -a;
            if (a >= n) a = 2 * (n - 1) - a;
            v = audio[a];
        }
        xs[i] = v;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < kFrames * kFFT; i += kThreads) {
        const int fr = i / kFFT, t = i % kFFT;
        xw[fr][t] = xs[fr * kHop + t] * win[t];  // float32 product, as the reference's frames * window
    }
    __syncthreads();
    // DFT bins: thread t takes (frame, bin) pairs t, t + 256, ...
    for (int q = threadIdx.x; q < kFrames * kBins; q += kThreads) {
        const int fr = q / kBins, k = q % kBins;
        float re = 0.f, im = 0.f;
        if (f0 + fr < n_frames) {
            const float* x = xw[fr];
            int j = 0;  // (k * t) mod 400, advanced incrementally
#pragma unroll 4
            for (int t = 0; t < kFFT; t++) {
                const float s = x[t];
                const float2 c = tw[j];
                re = fmaf(s, c.x, re);
                im = fmaf(-s, c.y, im);
                j += k;
                if (j >= kFFT) j -= kFFT;
            }
        }
        pw[fr][k] = re * re + im * im;
    }
    __syncthreads();
    // mel rows: thread t takes mel m = t % 128 for frames t / 128, + 2, ...
    float mx = -INFINITY;
    for (int q = threadIdx.x; q < kFrames * kMel; q += kThreads) {
        const int fr = q / kMel, m = q % kMel;
        if (f0 + fr >= n_frames) continue;
        float acc = 0.f;
        for (int k = 0; k < kBins; k++) acc = fmaf(__ldg(filters + (size_t)k * kMel + m), pw[fr][k], acc);
        const float lg = log10f(fmaxf(acc, 1e-10f));
        work[(size_t)(f0 + fr) * kMel + m] = lg;
        mx = fmaxf(mx, lg);
    }
    mx = b2::warp_max(mx);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = b2::float_order(mx);
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned m = 0;
        for (int i = 0; i < kThreads / 32; i++) m = red[i] > m ? red[i] : m;
        atomicMax(gmax, m);
    }
}

// out[m][t] = (max(v, gmax - 8) + 4) / 4 for the first T frames
__global__ void log_mel_finish(const float* __restrict__ work, const unsigned* __restrict__ gmax, int T,
                               float* __restrict__ out) {
    const float lo = ordered_max_decode(*gmax) - 8.0f;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= T * kMel) return;
    const int m = i / T, t = i % T;
    out[i] = (fmaxf(work[(size_t)t * kMel + m], lo) + 4.0f) / 4.0f;
}

__global__ void build_embed_rows(const float* __restrict__ table, int H, const int* __restrict__ pre, int n_pre,
                                 const float* __restrict__ audio, int n_audio, const int* __restrict__ suf,
                                 float* __restrict__ out) {
    const int r = blockIdx.x;
    const float* src;
    if (r < n_pre) src = table + (size_t)pre[r] * H;
    else if (r < n_pre + n_audio) src = audio + (size_t)(r - n_pre) * H;
    else src = table + (size_t)suf[r - n_pre - n_audio] * H;
    float* dst = out + (size_t)r * H;
    for (int i = threadIdx.x; i < H; i += blockDim.x) dst[i] = src[i];
}

}  // namespace

extern "C" size_t b2_log_mel_workspace(int n_samples) {
    if (n_samples <= kFFT / 2) return 0;
    const size_t frames = (size_t)(n_samples / kHop) + 1;
    return kMelWork + frames * kMel * 4;
}

extern "C" int b2_log_mel(const float* audio, int n_samples, const float* filters, float* out, void* work,
                          b2_stream_t stream) {
    if (!audio || !filters || !out || !work || n_samples <= kFFT / 2)
        return b2_set_error(B2_ERR_INVALID_ARG, "b2_log_mel: bad arguments (n=%d; needs > %d samples)", n_samples,
                            kFFT / 2);
    cudaStream_t s = (cudaStream_t)stream;
    const int n_frames = n_samples / kHop + 1, T = n_samples / kHop;
    unsigned char* w = static_cast<unsigned char*>(work);
    unsigned* gmax = reinterpret_cast<unsigned*>(w);
    float* logs = reinterpret_cast<float*>(w + kMelWork);
    B2_TRY(cudaMemsetAsync(gmax, 0, 4, s));  // below every key
    log_mel_frames<<<(n_frames + kFrames - 1) / kFrames, kThreads, 0, s>>>(audio, n_samples, n_frames, filters, logs,
                                                                           gmax);
    B2_TRY(cudaGetLastError());
    if (T > 0) {
        log_mel_finish<<<(T * kMel + 255) / 256, 256, 0, s>>>(logs, gmax, T, out);
        B2_TRY(cudaGetLastError());
    }
    return 0;
}

extern "C" int b2_build_embed(const float* table, int V, int H, const int* prefix_ids, int n_pre, const float* audio,
                              int n_audio, const int* suffix_ids, int n_suf, float* out, b2_stream_t stream) {
    if (!table || !out || V <= 0 || H <= 0 || n_pre < 0 || n_audio < 0 || n_suf < 0 ||
        (n_pre && !prefix_ids) || (n_audio && !audio) || (n_suf && !suffix_ids))
        return b2_set_error(B2_ERR_INVALID_ARG, "b2_build_embed: bad arguments");
    const int total = n_pre + n_audio + n_suf;
    if (total == 0) return 0;
    build_embed_rows<<<total, 256, 0, (cudaStream_t)stream>>>(table, H, prefix_ids, n_pre, audio, n_audio,
                                                              suffix_ids, out);
    B2_TRY(cudaGetLastError());
    return 0;
}
