// k_hift_dsp.cu — the HiFT vocoder's host DSP either side of the Snake stack,
// on the device:
//
//   cbx_nsf_source   HiFTVocoder::generate_source (hift_vocoder.cpp:853-965):
//                    f0 -> harmonic source s[t] (SineGen + SourceModuleHnNSF)
//   cbx_stft         stft_centered_host (hift_vocoder.cpp:465-498), the source
//                    STFT that feeds the source-downsampling convolutions
//   cbx_istft_post   the output tail (hift_vocoder.cpp:787-829): conv_post
//                    channels -> magnitude / phase -> istft_centered_host
//                    (:501-541) -> clamp to +-audio_limit
//
// All three are f32 in, f32 out and follow the engine's arithmetic: the f32
// roundings of its float expressions are kept (__fmul_rn / __fadd_rn, no FMA
// contraction), and its double sums stay double.
//
// NSF source.  The engine accumulates each harmonic's phase in double, one
// sample at a time: cs += f*(h+1)/sr (hift_vocoder.cpp:931-933).  A parallel
// prefix sum would round differently, and over a 10 s utterance the engine's
// sequential rounding drifts by up to ~4e-7 turns, enough to move the output
// by ~1e-6.  So the kernel replays the engine's sequential sum exactly, in
// closed form.  Let x be a positive double in the binade [2^e, 2^(e+1)), a
// multiple of u = 2^(e-52), and d >= 0 with q = d/u not a tie (frac(q) !=
// 1/2).  While every partial result stays inside that binade,
// fl(x + d) = x + RN(q)*u, so n sequential adds equal one integer
// multiply-add on the 53-bit mantissa: X + n*RN(q), X = x/u.  advance()
// applies that run by run and single-steps across binade boundaries and ties
// (a few dozen times per utterance in total).  A CTA reconstructs the exact
// running sum at the start of each of its frames from frame 0: a warp per
// harmonic scans 128 frames per step with an int64 warp prefix sum, and falls
// back to per-frame advance() where a chunk crosses a binade.  Inside a frame
// the increment is constant, so consecutive samples' phases differ by a
// fixed angle: each lane takes one double sincos at its first sample and then
// rotates (sin, cos) by the 32-sample angle in double, 4 DFMA-class ops per
// (sample, harmonic) instead of a double sin.  No scratch memory: every CTA
// recomputes its prefix from f0 (a few KB, L2-resident).
//
// STFT / iSTFT.  n_fft even, 2..32; twiddles are formed on the device with
// sincospi of the reduced angle 2*(k*n mod N)/N.  The STFT is a direct DFT
// per (frame, bin) in double over the f32 windowed frame (the engine's naive
// DFT); the iSTFT folds the n / N-n pairs of the inverse DFT (same cosine,
// opposite sine) and runs the overlap-add, window-square normalisation, trim
// and clamp in f32 in the engine's frame order.
#include <math.h>

#include "cbx_common.cuh"

namespace cbx {
namespace {

// ------------------------------------------------------------- NSF source --

constexpr int kHarm = CBX_NSF_HARMONICS;  // fundamental + 8 overtones
constexpr int kNsfThreads = 32 * kHarm;   // one warp per harmonic in the prologue
constexpr int kFpl = 4;                   // frames per lane per prologue step
constexpr int kPiece = 512;               // samples per warp per body pass (16 per lane)
constexpr float kSineAmp = 0.1f;          // SINE_AMP, hift_vocoder.cpp:859
constexpr float kNoiseStd = 0.003f;       // NOISE_STD, :860
constexpr float kVoicedThr = 10.0f;       // VOICED_THR, :861
constexpr double kTwoPi = 2.0 * 3.14159265358979323846;
constexpr double kTwo53 = 9007199254740992.0;
constexpr long long kMant = (1LL << 53) - 1;  // largest mantissa of a binade

struct NsfArgs {
    const float* f0;     // [B][n_mel]
    const float* phase;  // [B][9]
    const float* noise;  // [B][9][T]
    float* out;          // [B][T]
    int64_t n_mel;
    int64_t T;
    int up;
    int frames_per_cta;
    double inv_sr;
    float lw[kHarm];
    float lb;
};

// x = X * u with X the 53-bit mantissa (implicit bit included) and u = 2^(e-52).
// Valid for 2^-970 <= x < inf (so that 1/u is a normal double).
struct Binade {
    long long X;
    double u, inv_u;
};
__device__ __forceinline__ Binade binade_of(double x) {
    const long long bits = __double_as_longlong(x);
    const int be = (int)((bits >> 52) & 0x7FF);  // biased exponent of x
    Binade r;
    r.X = (bits & ((1LL << 52) - 1)) | (1LL << 52);
    r.u = __longlong_as_double((long long)(be - 52) << 52);       // 2^(e-52)
    r.inv_u = __longlong_as_double((long long)(2098 - be) << 52);  // 2^(52-e)
    return r;
}
__device__ __forceinline__ bool runs_ok(double x) { return x >= 0x1p-970 && x < kTwo53 * 0x1p+900; }

// Result of n sequential IEEE additions x = fl(x + d) (n >= 1), exactly.
__device__ double advance(double x, double d, long long n) {
    if (n <= 0) return x;
    if (!isfinite(x) || !isfinite(d) || d == 0.0) return __dadd_rn(x, d);  // constant after one add
    bool neg = false;
    if (d < 0.0) {
        if (x > 0.0) {  // magnitude shrinking through binades: plain adds (f0 < 0 only)
            for (; n > 0; --n) x = __dadd_rn(x, d);
            return x;
        }
        neg = true;  // round-to-nearest-even is symmetric: mirror to x >= 0, d > 0
        x = -x;
        d = -d;
    }
    while (n > 0) {
        if (runs_ok(x)) {
            const Binade bn = binade_of(x);
            const double q = d * bn.inv_u;  // exact: power-of-two scaling
            if (q < kTwo53) {
                const double fq = floor(q);
                if (q - fq != 0.5) {
                    const long long dn = (long long)rint(q);
                    if (dn == 0) break;  // d < u/2: fl(x + d) == x from here on
                    long long k = (kMant - bn.X) / dn;
                    if (k > 0) {
                        if (k > n) k = n;
                        x = (double)(bn.X + k * dn) * bn.u;
                        n -= k;
                        continue;
                    }
                }
            }
        }
        x = __dadd_rn(x, d);  // one step across a binade boundary (or a tie)
        --n;
    }
    return neg ? -x : x;
}

// Per-harmonic phase increment of frame f0 value `f`, in the engine's order:
// (double)f * (h + 1) * inv_sr (hift_vocoder.cpp:931).
__device__ __forceinline__ double increment(float f, int h, double inv_sr) {
    return __dmul_rn(__dmul_rn((double)f, (double)(h + 1)), inv_sr);
}

// Inclusive warp prefix sum of int64 values.
__device__ __forceinline__ long long warp_scan_incl(long long v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const long long t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
    }
    return v;
}

// Frame-start running sums: warp h reconstructs cs_h at the start of every
// frame m < m_end and stores those of frames [m0, m_end) in xs[h][m - m0].
__device__ void nsf_prologue(const NsfArgs& a, const float* f0b, int64_t m0, int64_t m_end,
                             double* xs_h) {
    const int h = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    double x = 0.0;  // cs before the first sample
    for (int64_t mb = 0; mb < m_end; mb += 32 * kFpl) {
        double dl[kFpl];
        long long pre[kFpl];
        long long sum = 0;
        const bool xok = runs_ok(x);
        const Binade bn = binade_of(xok ? x : 1.0);
        bool ok = xok;
#pragma unroll
        for (int i = 0; i < kFpl; ++i) {
            const int64_t m = mb + lane * kFpl + i;
            const bool valid = m < m_end;
            const double d = increment(valid ? __ldg(f0b + m) : 0.0f, h, a.inv_sr);
            dl[i] = d;
            pre[i] = sum;
            if (valid && ok) {
                const double q = d * bn.inv_u;
                // d >= 0 (also rejects NaN), no tie, and up * RN(q) kept far from overflow
                if (!(d >= 0.0) || !(q * (double)a.up < kTwo53) || q - floor(q) == 0.5) {
                    ok = false;
                } else {
                    sum += (long long)rint(q) * a.up;
                }
            }
        }
        const long long incl = warp_scan_incl(sum);
        const long long total = __shfl_sync(0xffffffffu, incl, 31);
        const bool fast = __all_sync(0xffffffffu, ok) && bn.X + total <= kMant;
        if (fast) {
            const long long excl = incl - sum;
#pragma unroll
            for (int i = 0; i < kFpl; ++i) {
                const int64_t m = mb + lane * kFpl + i;
                if (m >= m0 && m < m_end) xs_h[m - m0] = (double)(bn.X + excl + pre[i]) * bn.u;
            }
            x = (double)(bn.X + total) * bn.u;
        } else {
            // frame by frame (uniform across the warp)
            for (int src = 0; src < 32; ++src) {
#pragma unroll
                for (int i = 0; i < kFpl; ++i) {
                    const int64_t m = mb + src * kFpl + i;
                    const double d = __shfl_sync(0xffffffffu, dl[i], src);
                    if (m < m_end) {
                        if (m >= m0 && lane == 0) xs_h[m - m0] = x;
                        x = advance(x, d, a.up);
                    }
                }
            }
        }
    }
}

// Grid (ctas per utterance, B); 9 warps.  The CTA owns frames
// [m0, m0 + frames_per_cta); warp w computes frames m0 + w, m0 + w + 9, ...
__global__ void __launch_bounds__(kNsfThreads, 2) k_nsf_source(NsfArgs a) {
    extern __shared__ double xs[];  // [kHarm][frames_per_cta]
    const int64_t b = blockIdx.y;
    const int64_t m0 = (int64_t)blockIdx.x * a.frames_per_cta;
    int64_t m_end = m0 + a.frames_per_cta;
    if (m_end > a.n_mel) m_end = a.n_mel;
    const float* f0b = a.f0 + b * a.n_mel;
    grid_dep_wait();
    grid_dep_launch();
    if (m0 >= m_end) return;
    const int w = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    nsf_prologue(a, f0b, m0, m_end, xs + (int64_t)w * a.frames_per_cta);
    __syncthreads();

    float ph[kHarm];
#pragma unroll
    for (int h = 0; h < kHarm; ++h) ph[h] = h == 0 ? 0.0f : __ldg(a.phase + b * kHarm + h);
    const float namp_unvoiced = kSineAmp / 3.0f;

    for (int64_t m = m0 + w; m < m_end; m += kHarm) {
        const float f = __ldg(f0b + m);
        const float uv = (f > kVoicedThr) ? 1.0f : 0.0f;
        const float namp =
            __fadd_rn(__fmul_rn(uv, kNoiseStd), __fmul_rn(__fsub_rn(1.0f, uv), namp_unvoiced));
        const int64_t t_frame = m * a.up;
        for (int base = 0; base < a.up; base += kPiece) {
            double acc[kPiece / 32];
#pragma unroll
            for (int r = 0; r < kPiece / 32; ++r) acc[r] = (double)a.lb;
#pragma unroll 1
            for (int h = 0; h < kHarm; ++h) {
                const float* nz = a.noise + (b * kHarm + h) * a.T + t_frame;
                float nv[kPiece / 32];
#pragma unroll
                for (int r = 0; r < kPiece / 32; ++r) {
                    const int j = base + lane + 32 * r;
                    nv[r] = j < a.up ? __ldg(nz + j) : 0.0f;
                }
                const double xm = xs[(int64_t)h * a.frames_per_cta + (m - m0)];
                const double d = increment(f, h, a.inv_sr);
                // Is this frame one constant-increment run from xm?  Then
                // cs after s adds = (X + s*Dn) * u for every s <= up.
                bool run = false;
                long long X = 0, dn = 0;
                double u = 0.0;
                if (d == 0.0 && xm >= 0.0) {
                    run = true;  // cs stays xm (+0 for a -0 start: same phase)
                    X = 0;
                    u = 0.0;
                } else if (runs_ok(xm) && d > 0.0) {
                    const Binade bn = binade_of(xm);
                    const double q = d * bn.inv_u;
                    if (q < kTwo53 && q - floor(q) != 0.5) {
                        dn = (long long)rint(q);
                        X = bn.X;
                        u = bn.u;
                        run = dn == 0 || (kMant - X) / dn >= a.up;
                    }
                }
                const float lwh = a.lw[h];
                const double phd = (double)ph[h];
                if (run) {
                    // first sample of this lane: s0 = j + 1 adds into the frame
                    const long long s0 = base + lane + 1;
                    const double cs0 = d == 0.0 ? __dadd_rn(xm, d) : (double)(X + s0 * dn) * u;
                    const double th0 = __dadd_rn(__dmul_rn(kTwoPi, cs0 - floor(cs0)), phd);
                    double sn, cn, sw, cw;
                    sincos(th0, &sn, &cn);
                    const double inc = (double)(32 * dn) * u;  // 32 samples of phase, exact
                    sincospi(2.0 * (inc - floor(inc)), &sw, &cw);
#pragma unroll
                    for (int r = 0; r < kPiece / 32; ++r) {
                        const float sine = __fmul_rn(kSineAmp, __double2float_rn(sn));
                        const float sth = __fadd_rn(__fmul_rn(sine, uv), __fmul_rn(namp, nv[r]));
                        acc[r] = __dadd_rn(acc[r], (double)__fmul_rn(lwh, sth));
                        const double s2 = fma(sn, cw, cn * sw);
                        cn = fma(cn, cw, -(sn * sw));
                        sn = s2;
                    }
                } else {
                    // a binade boundary (or a tie) inside the frame: per sample
#pragma unroll 1
                    for (int r = 0; r < kPiece / 32; ++r) {
                        const int j = base + lane + 32 * r;
                        if (j >= a.up) break;
                        const double cs = advance(xm, d, j + 1);
                        const double th = __dadd_rn(__dmul_rn(kTwoPi, cs - floor(cs)), phd);
                        const float sine = __fmul_rn(kSineAmp, __double2float_rn(sin(th)));
                        const float sth = __fadd_rn(__fmul_rn(sine, uv), __fmul_rn(namp, nv[r]));
                        acc[r] = __dadd_rn(acc[r], (double)__fmul_rn(lwh, sth));
                    }
                }
            }
            float* o = a.out + b * a.T + t_frame;
#pragma unroll
            for (int r = 0; r < kPiece / 32; ++r) {
                const int j = base + lane + 32 * r;
                if (j < a.up) o[j] = tanhf(__double2float_rn(acc[r]));
            }
        }
    }
}

// ------------------------------------------------------------ STFT / iSTFT --

constexpr int kMaxFft = 32;
constexpr int kDspThreads = 256;

// cos / sin of 2 pi k n / N (sign of the forward transform applied by the caller)
__device__ __forceinline__ void twiddle(int k, int n, int N, double* c, double* s) {
    sincospi(2.0 * (double)((k * n) % N) / (double)N, s, c);
}

struct StftArgs {
    const float* x;  // [B][T]
    const float* window;
    float* out;
    int64_t T, Ts;
    int N, hop, layout, frames_per_cta;
};

// Reflect padding by N/2 about the edge samples (hift_vocoder.cpp:473-476).
__device__ __forceinline__ float padded_sample(const float* x, int64_t T, int pad, int64_t i) {
    if (i < pad) return __ldg(x + (pad - i));
    if (i >= pad + T) return __ldg(x + (T - 2 - (i - pad - T)));
    return __ldg(x + (i - pad));
}

// Grid (frame tiles, B).  Shared: twiddles [nb][N] (cos, sin), window [N],
// the tile's samples [(F-1)*hop + N].
__global__ void __launch_bounds__(kDspThreads) k_stft(StftArgs a) {
    extern __shared__ double sm[];
    const int N = a.N, nb = N / 2 + 1, pad = N / 2;
    double* tc = sm;            // [nb][N]
    double* ts = tc + nb * N;   // [nb][N]
    float* win = reinterpret_cast<float*>(ts + nb * N);
    float* smp = win + kMaxFft;
    const int64_t b = blockIdx.y;
    const int64_t t0 = (int64_t)blockIdx.x * a.frames_per_cta;
    int F = a.frames_per_cta;
    if (t0 + F > a.Ts) F = (int)(a.Ts - t0);
    const int ns = (F - 1) * a.hop + N;
    for (int i = threadIdx.x; i < nb * N; i += blockDim.x) twiddle(i / N, i % N, N, tc + i, ts + i);
    grid_dep_wait();
    grid_dep_launch();
    const float* xb = a.x + b * a.T;
    for (int i = threadIdx.x; i < N; i += blockDim.x) win[i] = __ldg(a.window + i);
    for (int i = threadIdx.x; i < ns; i += blockDim.x)
        smp[i] = padded_sample(xb, a.T, pad, t0 * a.hop + i);
    __syncthreads();
    const int items = F * nb;
    for (int it = threadIdx.x; it < items; it += blockDim.x) {
        // BTC: bins of a frame on consecutive threads; BCT: frames of a bin
        const int f = a.layout == CBX_LAYOUT_BTC ? it / nb : it % F;
        const int k = a.layout == CBX_LAYOUT_BTC ? it % nb : it / F;
        const float* fr = smp + f * a.hop;
        double re = 0.0, im = 0.0;
        for (int n = 0; n < N; ++n) {
            const double v = (double)__fmul_rn(fr[n], win[n]);  // frame[n] = x * window in f32
            re = fma(v, tc[k * N + n], re);
            im = fma(-v, ts[k * N + n], im);  // e^{-i a}
        }
        const int64_t t = t0 + f;
        if (a.layout == CBX_LAYOUT_BTC) {
            float* o = a.out + (b * a.Ts + t) * 2 * nb;
            o[k] = __double2float_rn(re);
            o[nb + k] = __double2float_rn(im);
        } else {
            a.out[(b * 2 * nb + k) * a.Ts + t] = __double2float_rn(re);
            a.out[(b * 2 * nb + nb + k) * a.Ts + t] = __double2float_rn(im);
        }
    }
}

struct IstftArgs {
    const float* post;  // BTC [B][Tf][2 nb] or BCT [B][2 nb][Tf]
    const float* window;
    float* out;  // [B][Ta]
    int64_t Tf, Ta;
    int N, hop, layout, samples_per_cta;
    float limit;
};

// Grid (output tiles, B).  A tile of S output samples (padded positions
// P0 + pad .. ) needs frames [f_lo, f_hi]; shared holds their spectra
// (re, im f32) and windowed inverse frames (f32), then each thread sums one
// output sample over its frames in ascending frame order.
__global__ void __launch_bounds__(kDspThreads) k_istft_post(IstftArgs a) {
    extern __shared__ double sm[];
    const int N = a.N, nb = N / 2 + 1, pad = N / 2, hop = a.hop;
    double* tc = sm;           // [nb][N]
    double* ts = tc + nb * N;  // [nb][N]
    float* win = reinterpret_cast<float*>(ts + nb * N);
    const int64_t b = blockIdx.y;
    const int64_t i0 = (int64_t)blockIdx.x * a.samples_per_cta;  // first output sample
    int S = a.samples_per_cta;
    if (i0 + S > a.Ta) S = (int)(a.Ta - i0);
    const int64_t p_lo = i0 + pad, p_hi = i0 + pad + S - 1;  // padded positions
    int64_t f_lo = p_lo - N + 1 > 0 ? (p_lo - N + 1 + hop - 1) / hop : 0;
    int64_t f_hi = p_hi / hop;
    if (f_hi > a.Tf - 1) f_hi = a.Tf - 1;
    const int nf = (int)(f_hi - f_lo + 1);
    const int max_nf = (a.samples_per_cta + N - 2) / hop + 2;
    float* re = win + kMaxFft;            // [max_nf][nb]
    float* im = re + max_nf * nb;         // [max_nf][nb]
    float* fr = im + max_nf * nb;         // [max_nf][N]  windowed inverse frames
    for (int i = threadIdx.x; i < nb * N; i += blockDim.x) twiddle(i / N, i % N, N, tc + i, ts + i);
    grid_dep_wait();
    grid_dep_launch();
    for (int i = threadIdx.x; i < N; i += blockDim.x) win[i] = __ldg(a.window + i);
    // 1. magnitude / phase -> (re, im) per (frame, bin), f32 as the engine
    for (int it = threadIdx.x; it < nf * nb; it += blockDim.x) {
        const int f = a.layout == CBX_LAYOUT_BTC ? it / nb : it % nf;
        const int k = a.layout == CBX_LAYOUT_BTC ? it % nb : it / nf;
        const int64_t t = f_lo + f;
        float mraw, praw;
        if (a.layout == CBX_LAYOUT_BTC) {
            const float* p = a.post + (b * a.Tf + t) * 2 * nb;
            mraw = __ldg(p + k);
            praw = __ldg(p + nb + k);
        } else {
            mraw = __ldg(a.post + (b * 2 * nb + k) * a.Tf + t);
            praw = __ldg(a.post + (b * 2 * nb + nb + k) * a.Tf + t);
        }
        const float e = expf(mraw);
        const float mag = (100.0f < e) ? 100.0f : e;  // std::min(exp(raw), 100.0f)
        const float phs = sinf(praw);
        float sp, cp;
        sincosf(phs, &sp, &cp);
        re[f * nb + k] = __fmul_rn(mag, cp);
        im[f * nb + k] = __fmul_rn(mag, sp);
    }
    __syncthreads();
    // 2. inverse DFT per (frame, n-pair) in double; frame[n] = x_n / N in f32, times window
    const int half = N / 2;
    for (int it = threadIdx.x; it < nf * (half + 1); it += blockDim.x) {
        const int f = it / (half + 1), n = it % (half + 1);
        const float* rf = re + f * nb;
        const float* imf = im + f * nb;
        double A = (double)rf[0] + ((n & 1) ? -(double)rf[nb - 1] : (double)rf[nb - 1]);
        double Bs = 0.0;
        for (int k = 1; k < nb - 1; ++k) {
            A = fma(2.0 * (double)rf[k], tc[k * N + n], A);
            Bs = fma(2.0 * (double)imf[k], ts[k * N + n], Bs);
        }
        fr[f * N + n] = __fmul_rn(__double2float_rn(__ddiv_rn(A - Bs, (double)N)), win[n]);
        if (n != 0 && n != half)
            fr[f * N + (N - n)] =
                __fmul_rn(__double2float_rn(__ddiv_rn(A + Bs, (double)N)), win[N - n]);
    }
    __syncthreads();
    // 3. overlap-add in frame order, window-square normalisation, clamp
    for (int i = threadIdx.x; i < S; i += blockDim.x) {
        const int64_t p = i0 + pad + i;
        int64_t t = p - N + 1 > 0 ? (p - N + 1 + hop - 1) / hop : 0;
        float acc = 0.0f, wsum = 0.0f;
        for (; t <= f_hi && t * hop <= p; ++t) {
            const int n = (int)(p - t * hop);
            acc = __fadd_rn(acc, fr[(t - f_lo) * N + n]);
            wsum = __fadd_rn(wsum, __fmul_rn(win[n], win[n]));
        }
        if (wsum > 1e-11f) acc = __fdiv_rn(acc, wsum);
        const float lim = a.limit;
        a.out[b * a.Ta + i0 + i] = (acc < -lim) ? -lim : ((lim < acc) ? lim : acc);
    }
}

size_t dsp_twiddle_bytes(int N) { return 2 * (size_t)(N / 2 + 1) * N * sizeof(double) + kMaxFft * 4; }

}  // namespace
}  // namespace cbx

using namespace cbx;

extern "C" {

// HiFTVocoder::generate_source, hift_vocoder.cpp:853-965 (phase_vec_opt and
// noise_z_opt given).
CBX_API int cbx_nsf_source(const float* f0, int64_t B, int64_t n_mel, int32_t upsample,
                           int32_t sampling_rate, const float* phase, const float* noise,
                           const float* lin_w_host, float lin_b, float* out, cbx_stream_t stream) {
    if (B < 0 || n_mel < 0) return fail(CBX_ERR_INVALID_ARG, "cbx_nsf_source: B or n_mel < 0");
    if (upsample <= 0 || sampling_rate <= 0)
        return fail(CBX_ERR_INVALID_ARG, "cbx_nsf_source: upsample %d / sampling_rate %d must be > 0",
                    upsample, sampling_rate);
    if (B == 0 || n_mel == 0) return ok();
    if (!f0 || !phase || !noise || !lin_w_host || !out)
        return fail(CBX_ERR_INVALID_ARG, "cbx_nsf_source: NULL pointer");
    if (n_mel > ((int64_t)1 << 40) / upsample)
        return fail(CBX_ERR_INVALID_ARG, "cbx_nsf_source: n_mel * upsample too large");
    NsfArgs a;
    a.f0 = f0;
    a.phase = phase;
    a.noise = noise;
    a.out = out;
    a.n_mel = n_mel;
    a.T = n_mel * upsample;
    a.up = upsample;
    a.inv_sr = 1.0 / (double)sampling_rate;
    for (int h = 0; h < kHarm; ++h) a.lw[h] = lin_w_host[h];
    a.lb = lin_b;
    // frames per CTA: a multiple of the 9 warps, about two waves of CTAs
    const int64_t frames = B * n_mel;
    const int64_t target = (int64_t)num_sms() * 2 * 2;
    int64_t fpc = kHarm * ((frames + target * kHarm - 1) / (target * kHarm));
    if (fpc < kHarm) fpc = kHarm;
    if (fpc > 8 * kHarm) fpc = 8 * kHarm;
    a.frames_per_cta = (int)fpc;
    const int64_t ctas = (n_mel + fpc - 1) / fpc;
    if (B > 65535) return fail(CBX_ERR_INVALID_ARG, "cbx_nsf_source: B > 65535");
    const size_t smem = (size_t)kHarm * fpc * sizeof(double);
    return launch_status(launch(k_nsf_source, dim3((unsigned)ctas, (unsigned)B), dim3(kNsfThreads),
                                smem, stream, a),
                         "cbx_nsf_source");
}

// stft_centered_host, hift_vocoder.cpp:465-498.
CBX_API int cbx_stft(const float* audio, int64_t B, int64_t T, int32_t n_fft, int32_t hop,
                     const float* window, int layout, float* out, cbx_stream_t stream) {
    if (n_fft < 2 || n_fft > kMaxFft || (n_fft & 1))
        return fail(CBX_ERR_INVALID_ARG, "cbx_stft: n_fft %d must be even, 2..%d", n_fft, kMaxFft);
    if (hop < 1 || hop > n_fft)
        return fail(CBX_ERR_INVALID_ARG, "cbx_stft: hop %d outside 1..n_fft", hop);
    if (layout != CBX_LAYOUT_BCT && layout != CBX_LAYOUT_BTC)
        return fail(CBX_ERR_INVALID_ARG, "cbx_stft: bad layout %d", layout);
    if (B < 0) return fail(CBX_ERR_INVALID_ARG, "cbx_stft: B < 0");
    if (B == 0) return ok();
    if (T <= n_fft / 2)
        return fail(CBX_ERR_INVALID_ARG, "cbx_stft: T %lld must exceed n_fft / 2 (reflect padding)",
                    (long long)T);
    if (!audio || !window || !out) return fail(CBX_ERR_INVALID_ARG, "cbx_stft: NULL pointer");
    if (B > 65535) return fail(CBX_ERR_INVALID_ARG, "cbx_stft: B > 65535");
    StftArgs a;
    a.x = audio;
    a.window = window;
    a.out = out;
    a.T = T;
    a.Ts = 1 + T / hop;  // 1 + (T + 2 pad - n_fft) / hop with pad = n_fft / 2
    a.N = n_fft;
    a.hop = hop;
    a.layout = layout;
    a.frames_per_cta = 256;
    const size_t smem =
        dsp_twiddle_bytes(n_fft) + (size_t)((a.frames_per_cta - 1) * hop + n_fft) * sizeof(float);
    const int64_t tiles = (a.Ts + a.frames_per_cta - 1) / a.frames_per_cta;
    return launch_status(
        launch(k_stft, dim3((unsigned)tiles, (unsigned)B), dim3(kDspThreads), smem, stream, a),
        "cbx_stft");
}

// HiFT output tail, hift_vocoder.cpp:787-829 (istft_centered_host :501-541).
CBX_API int cbx_istft_post(const float* post, int64_t B, int64_t n_frames, int32_t n_fft,
                           int32_t hop, const float* window, int layout, float audio_limit,
                           float* out, cbx_stream_t stream) {
    if (n_fft < 2 || n_fft > kMaxFft || (n_fft & 1))
        return fail(CBX_ERR_INVALID_ARG, "cbx_istft_post: n_fft %d must be even, 2..%d", n_fft,
                    kMaxFft);
    if (hop < 1 || hop > n_fft)
        return fail(CBX_ERR_INVALID_ARG, "cbx_istft_post: hop %d outside 1..n_fft", hop);
    if (layout != CBX_LAYOUT_BCT && layout != CBX_LAYOUT_BTC)
        return fail(CBX_ERR_INVALID_ARG, "cbx_istft_post: bad layout %d", layout);
    if (B < 0 || n_frames < 0) return fail(CBX_ERR_INVALID_ARG, "cbx_istft_post: B or n_frames < 0");
    if (!(audio_limit >= 0.0f))
        return fail(CBX_ERR_INVALID_ARG, "cbx_istft_post: audio_limit must be >= 0 (inf: no clamp)");
    if (B == 0 || n_frames <= 1) return ok();  // (n_frames - 1) * hop output samples
    if (!post || !window || !out) return fail(CBX_ERR_INVALID_ARG, "cbx_istft_post: NULL pointer");
    if (B > 65535) return fail(CBX_ERR_INVALID_ARG, "cbx_istft_post: B > 65535");
    IstftArgs a;
    a.post = post;
    a.window = window;
    a.out = out;
    a.Tf = n_frames;
    a.Ta = (n_frames - 1) * hop;
    a.N = n_fft;
    a.hop = hop;
    a.layout = layout;
    a.limit = audio_limit;
    // keep twiddles + the tile's spectra and frames within the default 48 KB
    const int nb = n_fft / 2 + 1;
    int S = 1024;
    auto tile_bytes = [&](int s) {
        const int max_nf = (s + n_fft - 2) / hop + 2;
        return (size_t)max_nf * (2 * nb + n_fft) * sizeof(float);
    };
    while (S > 64 && dsp_twiddle_bytes(n_fft) + tile_bytes(S) > 48 * 1024) S /= 2;
    a.samples_per_cta = S;
    const size_t smem = dsp_twiddle_bytes(n_fft) + tile_bytes(S);
    const int64_t tiles = (a.Ta + S - 1) / S;
    return launch_status(
        launch(k_istft_post, dim3((unsigned)tiles, (unsigned)B), dim3(kDspThreads), smem, stream, a),
        "cbx_istft_post");
}

// Periodic Hann window, the engine's f32 host expression
// (hift_vocoder.cpp:429-434).
CBX_API int cbx_hann_window(int32_t n_fft, float* window_host) {
    if (n_fft <= 0 || !window_host)
        return fail(CBX_ERR_INVALID_ARG, "cbx_hann_window: bad arguments");
    for (int32_t n = 0; n < n_fft; ++n)
        window_host[n] = 0.5f - 0.5f * cosf(2.0f * (float)3.14159265358979323846 * n / n_fft);
    return ok();
}

}  // extern "C"
