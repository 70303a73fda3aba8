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
// (a few dozen times per utterance in total).  The exact running sum at every
// frame start comes from one scan per (utterance, harmonic): a warp takes 128
// frames per step with an int64 warp prefix sum and falls back to per-frame
// advance() where a step crosses a binade.  k_nsf_phase_starts runs those
// scans first and parks each frame's 9 sums in that frame's own output
// samples, which the sample kernel reads back before writing them (no scratch
// memory); where they do not fit (odd or small upsample, misaligned output)
// each CTA replays its utterance up to its frames itself.  Inside a frame the
// increment is constant, so consecutive samples' phases differ by a fixed
// angle: each lane takes one double sincos at its first sample, one rotation
// for its second, and then the Chebyshev recurrence sin((k+1)t) =
// 2 cos t sin(kt) - sin((k-1)t): one DFMA per (sample, harmonic) instead of a
// double sin.
//
// STFT / iSTFT.  n_fft even, 2..32.  The STFT is a DFT per frame in double
// over the f32 windowed frame (the engine's naive DFT, folded over the n /
// N-n pairs); the iSTFT folds the n / N-n pairs of the inverse DFT (same
// cosine, opposite sine) and runs the overlap-add, window-square
// normalisation, trim and clamp in f32 in the engine's frame order.  The
// engine's sizes (n_fft 16, hop 4) and 8 / 2 run persistent kernels fed by
// bulk async copies with compile-time twiddles; other sizes and misaligned
// inputs run one tile per CTA with twiddles formed on the device by sincospi
// of the reduced angle 2*(k*n mod N)/N.
#include <math.h>
#include <stdlib.h>

#include "cbx_common.cuh"

namespace cbx {
namespace {

// ------------------------------------------------------------- NSF source --

constexpr int kHarm = CBX_NSF_HARMONICS;  // fundamental + 8 overtones
constexpr int kNsfWarps = 8;             // 2 per SM sub-partition
constexpr int kNsfThreads = 32 * kNsfWarps;
constexpr int kFpl = 4;                   // frames per lane per prologue step
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
    int64_t B;
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

// Largest k <= n with X + k * dn <= kMant (dn > 0, X <= kMant), without a
// division on the critical path: an f32 estimate room * (1 / dn) (relative
// error ~2^-22, so within one of the quotient while that is below 2^21; larger
// quotients exceed n and are capped), then exact int64 corrections.
__device__ __forceinline__ long long run_length(long long X, long long dn, long long n) {
    const long long room = kMant - X;
    if ((double)n * (double)dn < 0x1p+62 && n * dn <= room) return n;
    const float kf = __fmul_rn((float)room, __frcp_rn((float)dn));
    long long k = kf >= (float)n ? n : (long long)kf;
    while (k > 0 && X + k * dn > kMant) --k;
    while (k < n && X + (k + 1) * dn <= kMant) ++k;
    return k;
}

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
                    const long long k = run_length(bn.X, dn, n);
                    if (k > 0) {
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

// Frame-start running sums: warp h, given cs_h = x_start at the start of frame
// m_start, reconstructs cs_h at the start of every frame m_start <= m < m_end,
// stores those of frames [m0, m_end) in xs[h][m - m0] and returns cs_h at m_end.
// Each step takes the next 128 frames (4 per lane): with x in binade e, every
// frame contributes up * RN(d / u) mantissa units; an int64 warp prefix sum
// gives all frame starts at once, up to the first frame that leaves the
// binade (or has a tie, a negative or non-finite increment).  That frame is
// replayed by advance() and the next step starts after it.
// inc_sm: the harmonic's per-frame increments precomputed in shared memory
// (indexed by frame), or NULL to form them from f0b.
__device__ double nsf_prologue(const NsfArgs& a, int h, const float* f0b, int64_t m_start,
                               double x_start, int64_t m0, int64_t m_end, double* xs_h,
                               int64_t xs_stride = 1, const double* inc_sm = nullptr) {
    const int lane = threadIdx.x & 31;
    double x = x_start;  // cs before frame mb
    int64_t mb = m_start;
    while (mb < m_end) {
        const bool xok = runs_ok(x);
        const Binade bn = binade_of(xok ? x : 1.0);
        double dl[kFpl];
        long long cl[kFpl];  // mantissa units of each frame (0 when not a fast frame)
        int first_bad = kFpl;
        long long sum = 0;
#pragma unroll
        for (int i = 0; i < kFpl; ++i) {
            const int64_t m = mb + lane * kFpl + i;
            const bool valid = m < m_end;
            const double d = inc_sm ? (valid ? inc_sm[m] : 0.0)
                                    : increment(valid ? __ldg(f0b + m) : 0.0f, h, a.inv_sr);
            dl[i] = d;
            const double q = d * bn.inv_u;
            const bool fast = valid && xok && d >= 0.0 && q * (double)a.up < kTwo53 &&
                              q - floor(q) != 0.5;
            cl[i] = fast ? (long long)rint(q) * a.up : 0;
            if (!fast && first_bad == kFpl) first_bad = i;
            if (first_bad == kFpl) sum += cl[i];
        }
        const long long incl = warp_scan_incl(sum);
        const long long excl = incl - sum;
        // frames up to this lane's first bad one, cut where the binade overflows
        long long run = bn.X + excl;
        int lane_stop = first_bad;
#pragma unroll
        for (int i = 0; i < kFpl; ++i) {
            if (i < lane_stop) {
                if (run + cl[i] > kMant) lane_stop = i;
                else run += cl[i];
            }
        }
        // first stopping frame of the warp (index within the 128), or 128
        const int key = lane_stop < kFpl ? lane * kFpl + lane_stop : 32 * kFpl;
        const int g = (int)__reduce_min_sync(0xffffffffu, (unsigned)key);
        // frames before g: starts are X + prefix, stored in mantissa units
        {
            long long st = bn.X + excl;
#pragma unroll
            for (int i = 0; i < kFpl; ++i) {
                const int idx = lane * kFpl + i;
                const int64_t m = mb + idx;
                if (idx < g && m >= m0 && m < m_end) xs_h[(m - m0) * xs_stride] = (double)st * bn.u;
                st += cl[i];
            }
        }
        if (g == 32 * kFpl) {  // the whole step was one run
            x = (double)(__shfl_sync(0xffffffffu, incl, 31) + bn.X) * bn.u;
            mb += 32 * kFpl;
            continue;
        }
        const int64_t G = mb + g;
        // start of frame G and its increment, from the lane that owns it
        const int owner = g / kFpl, gi = g % kFpl;
        long long st = bn.X + excl;
        double dg = dl[0];
#pragma unroll
        for (int i = 0; i < kFpl; ++i) {
            if (i < gi) st += cl[i];
            if (i == gi) dg = dl[i];
        }
        const long long st_g = __shfl_sync(0xffffffffu, st, owner);
        dg = __shfl_sync(0xffffffffu, dg, owner);
        const double xg = g == 0 ? x : (double)st_g * bn.u;
        if (G >= m_end) {  // every frame before m_end was one run: xg is cs at m_end
            x = xg;
            break;
        }
        if (lane == 0 && G >= m0) xs_h[(G - m0) * xs_stride] = xg;
        x = advance(xg, dg, a.up);
        mb = G + 1;
    }
    return x;  // cs at the start of frame m_end
}

// Per (harmonic, frame) of the CTA, filled by the prologue warp of that
// harmonic with one lane per frame.  kind 1: the frame is one constant-step
// run from its start xm, cs after s adds = (X1 + s dn1) u1 for all s <= up
// (u1 == 0: d == 0, cs stays xm).  kind 2: the run covers k1 adds, add k1 + 1
// crosses into the next binade (its IEEE result xc is stored) and a second run
// (X2, dn2, u2) covers the rest.  kind 0 (several crossings, a tie, a zero
// start): the frame is walked add by add.  (cw, sw): the rotation by 32
// samples of phase within each run.
struct FrameRun {
    long long X1, dn1, X2, dn2;
    double u1, u2, xc, xm;
    double cw1, sw1, cw2, sw2;
    int k1, kind;
};

// One constant-step run from x for n adds of d (d > 0): its mantissa, step and
// unit, or false.
__device__ __forceinline__ bool run_of(double x, double d, int n, long long* X, long long* dn,
                                       double* u) {
    if (!runs_ok(x) || !(d > 0.0)) return false;
    const Binade bn = binade_of(x);
    const double q = d * bn.inv_u;
    if (!(q * (double)n < kTwo53) || q - floor(q) == 0.5) return false;
    *dn = (long long)rint(q);
    *X = bn.X;
    *u = bn.u;
    return true;
}

// The run table entry of frame m (harmonic h) from its start value xm.
__device__ void nsf_frame_entry(const NsfArgs& a, int h, const float* f0b, int64_t m, double xm,
                                FrameRun* out) {
    FrameRun fr;
    fr.xm = xm;
    const double d = increment(__ldg(f0b + m), h, a.inv_sr);
    fr.kind = 0;
    fr.X1 = fr.dn1 = fr.X2 = fr.dn2 = 0;
    fr.u1 = fr.u2 = 0.0;
    fr.xc = 0.0;
    fr.k1 = a.up;
    if (d == 0.0 && fr.xm >= 0.0) {
        fr.kind = 1;  // cs stays xm (+0 for a -0 start: same phase)
    } else if (run_of(fr.xm, d, a.up, &fr.X1, &fr.dn1, &fr.u1)) {
        if (fr.dn1 == 0 || fr.X1 + fr.dn1 * a.up <= kMant) {
            fr.kind = 1;
        } else {
            const int k1 = (int)run_length(fr.X1, fr.dn1, a.up);
            const double xk = (double)(fr.X1 + k1 * fr.dn1) * fr.u1;
            fr.xc = __dadd_rn(xk, d);  // the crossing add
            fr.k1 = k1;
            const int r2 = a.up - k1 - 1;
            if (r2 == 0) {
                fr.kind = 2;
            } else if (run_of(fr.xc, d, r2, &fr.X2, &fr.dn2, &fr.u2) &&
                       (fr.dn2 == 0 || fr.X2 + fr.dn2 * r2 <= kMant)) {
                fr.kind = 2;
            }
        }
    }
    double inc = (double)(32 * fr.dn1) * fr.u1;  // 32 samples of phase, exact
    sincospi(2.0 * (inc - floor(inc)), &fr.sw1, &fr.cw1);
    inc = (double)(32 * fr.dn2) * fr.u2;
    sincospi(2.0 * (inc - floor(inc)), &fr.sw2, &fr.cw2);
    *out = fr;
}

// cs after s adds into a kind-1/2 frame (1 <= s <= up).
__device__ __forceinline__ double frame_cs(const FrameRun& fr, long long s) {
    if (fr.u1 == 0.0 && fr.kind == 1) return __dadd_rn(fr.xm, 0.0);
    if (s <= fr.k1) return (double)(fr.X1 + s * fr.dn1) * fr.u1;
    if (s == fr.k1 + 1) return fr.xc;
    return (double)(fr.X2 + (s - fr.k1 - 1) * fr.dn2) * fr.u2;
}

// (sin, cos) of 2 pi frac(cs) + p from sincospi of the turn fraction and the
// harmonic's (sin p, cos p): the engine's sin(2 pi frac(cs) + p) without a
// double-precision range reduction.
__device__ __forceinline__ void phase_at(double cs, double sp, double cp, double* sn, double* cn) {
    double s1, c1;
    sincospi(2.0 * (cs - floor(cs)), &s1, &c1);
    *sn = fma(s1, cp, c1 * sp);
    *cn = fma(c1, cp, -(s1 * sp));
}

// The samples of frames [m0, m_end) of utterance b (see k_nsf_source).  SPL
// samples per lane per pass (32 SPL per warp); EXACT: up == 32 SPL, one pass
// with no per-sample bounds checks (the engine's upsample 480 = 32 x 15).
// Per (frame, harmonic) one of four loops runs, chosen per warp from the
// frame's run table:
//   constant   d == 0 (an unvoiced frame): cs stays xm, the phase is one value;
//   one run    kind 1: (sin, cos) rotated by the run's 32-sample angle;
//   two runs   kind 2: as one run, restarting at the lane's first sample past
//              the crossing add (sample index r_sw of the lane);
//   walk       kind 0: the engine's adds one by one.
template <int SPL, bool EXACT>
__device__ __forceinline__ void nsf_frames(const NsfArgs& a, int64_t b, const float* f0b,
                                           int64_t m0, int64_t m_end, const FrameRun* tb,
                                           const float* s_lw, const double* s_pc, int* next,
                                           int lane) {
    constexpr int kSpan = 32 * SPL;  // samples per warp per pass
    const int fpc = a.frames_per_cta;
    const float namp_unvoiced = kSineAmp / 3.0f;

    for (;;) {
        // frames are handed out one at a time (warps on a busier sub-partition
        // take fewer)
        int idx = 0;
        if (lane == 0) idx = atomicAdd(next, 1);
        idx = __shfl_sync(0xffffffffu, idx, 0);
        const int64_t m = m0 + idx;
        if (m >= m_end) break;
        const float f = __ldg(f0b + m);
        const float uv = (f > kVoicedThr) ? 1.0f : 0.0f;
        const float namp =
            __fadd_rn(__fmul_rn(uv, kNoiseStd), __fmul_rn(__fsub_rn(1.0f, uv), namp_unvoiced));
        const int64_t t_frame = m * a.up;
        // the frame's 9 noise rows into L2 (lane h: row h), so harmonic h + 1's
        // loads are L2 hits by the time harmonic h is done
        if (lane < kHarm) {
            const float* row = a.noise + (b * kHarm + lane) * a.T + t_frame;
            const uintptr_t s0 = (reinterpret_cast<uintptr_t>(row) + 15) & ~uintptr_t(15);
            const uintptr_t s1 = reinterpret_cast<uintptr_t>(row + a.up) & ~uintptr_t(15);
            if (s1 > s0) prefetch_l2(reinterpret_cast<const void*>(s0), (uint32_t)(s1 - s0));
        }
        for (int base = 0; base < a.up; base += kSpan) {
            double acc[SPL];
#pragma unroll
            for (int r = 0; r < SPL; ++r) acc[r] = (double)a.lb;
#pragma unroll 1
            for (int h = 0; h < kHarm; ++h) {
                const float* nz = a.noise + (b * kHarm + h) * a.T + t_frame + base + lane;
                float nv[SPL];
#pragma unroll
                for (int r = 0; r < SPL; ++r)
                    nv[r] = (EXACT || base + lane + 32 * r < a.up) ? __ldg(nz + 32 * r) : 0.0f;
                const FrameRun& fr = tb[h * fpc + (m - m0)];
                const float lwh = s_lw[h];
                const int kind = fr.kind;
                // sample r of this lane: sth = SINE_AMP sin(theta) uv + namp noise,
                // accumulated in double in harmonic order (hift_vocoder.cpp:935-958)
                auto add = [&](int r, double sn) {
                    const float sine = __fmul_rn(kSineAmp, __double2float_rn(sn));
                    const float sth = __fadd_rn(__fmul_rn(sine, uv), __fmul_rn(namp, nv[r]));
                    acc[r] = __dadd_rn(acc[r], (double)__fmul_rn(lwh, sth));
                };
                // samples r and r + 1 at once: the same f32 operations on packed
                // f32x2 instructions (the same roundings), the double adds apart
                auto add2 = [&](int r, double sn0, double sn1) {
                    const float2 sine = __fmul2_rn(make_float2(kSineAmp, kSineAmp),
                                                   make_float2(__double2float_rn(sn0),
                                                               __double2float_rn(sn1)));
                    const float2 sth = __fadd2_rn(__fmul2_rn(sine, make_float2(uv, uv)),
                                                  __fmul2_rn(make_float2(namp, namp),
                                                             make_float2(nv[r], nv[r + 1])));
                    const float2 w = __fmul2_rn(make_float2(lwh, lwh), sth);
                    acc[r] = __dadd_rn(acc[r], (double)w.x);
                    acc[r + 1] = __dadd_rn(acc[r + 1], (double)w.y);
                };
                if (kind != 0) {
                    const double sp = s_pc[2 * h], cp = s_pc[2 * h + 1];
                    // first sample of this lane: s0 = base + lane + 1 adds into the frame
                    const int s0 = base + lane + 1;
                    double sn, cn;
                    if (kind == 1 && fr.u1 == 0.0) {
                        phase_at(__dadd_rn(fr.xm, 0.0), sp, cp, &sn, &cn);
#pragma unroll
                        for (int r = 0; r + 1 < SPL; r += 2) add2(r, sn, sn);
                        if constexpr (SPL % 2) add(SPL - 1, sn);
                    } else if (kind == 1) {
                        // sin at the lane's samples r and r + 1, then the
                        // Chebyshev recurrence sin((k+1)t) = 2 cos t sin(kt) - sin((k-1)t)
                        // with t the run's 32-sample angle: one DFMA per sample
                        phase_at((double)(fr.X1 + (long long)s0 * fr.dn1) * fr.u1, sp, cp, &sn, &cn);
                        const double c2 = 2.0 * fr.cw1;
                        double sa = sn, sb = fma(sn, fr.cw1, cn * fr.sw1);
#pragma unroll
                        for (int r = 0; r + 1 < SPL; r += 2) {
                            add2(r, sa, sb);
                            const double t1 = fma(c2, sb, -sa);
                            const double t2 = fma(c2, t1, -sb);
                            sa = t1;
                            sb = t2;
                        }
                        if constexpr (SPL % 2) add(SPL - 1, sa);
                    } else {
                        // r_sw: the lane's first sample past the crossing add,
                        // where the recurrence restarts in the second run
                        const int k1 = fr.k1;
                        const bool first = s0 <= k1;
                        const int r_sw = first ? (k1 - s0) / 32 + 1 : SPL;
                        phase_at(frame_cs(fr, s0), sp, cp, &sn, &cn);
                        double cw = first ? fr.cw1 : fr.cw2, sw = first ? fr.sw1 : fr.sw2;
                        double c2 = 2.0 * cw;
                        double sa = sn, sb = fma(sn, cw, cn * sw);
#pragma unroll
                        for (int r = 0; r < SPL; ++r) {
                            if (r > 0 && r == r_sw) {
                                phase_at(frame_cs(fr, s0 + 32 * r), sp, cp, &sn, &cn);
                                c2 = 2.0 * fr.cw2;
                                sa = sn;
                                sb = fma(sn, fr.cw2, cn * fr.sw2);
                            }
                            add(r, sa);
                            const double t = fma(c2, sb, -sa);
                            sa = sb;
                            sb = t;
                        }
                    }
                } else {
                    // a binade boundary, a tie or a zero start inside the frame:
                    // the engine's adds one by one (uniform), each lane keeping
                    // the running sum after its own sample
                    const double phd = h == 0 ? 0.0 : (double)__ldg(a.phase + b * kHarm + h);
                    const double d = increment(f, h, a.inv_sr);
                    double cb = fr.xm;
                    for (int k = 0; k < base; ++k) cb = __dadd_rn(cb, d);
#pragma unroll
                    for (int r = 0; r < SPL; ++r) {
                        if (!EXACT && base + 32 * r >= a.up) break;  // uniform
                        double cs = cb;
                        for (int k = 0; k < 32; ++k) {
                            cb = __dadd_rn(cb, d);
                            if (k == lane) cs = cb;
                        }
                        if (EXACT || base + lane + 32 * r < a.up) {
                            const double th = __dadd_rn(__dmul_rn(kTwoPi, cs - floor(cs)), phd);
                            add(r, sin(th));
                        }
                    }
                }
            }
            float* o = a.out + b * a.T + t_frame + base + lane;
#pragma unroll
            for (int r = 0; r < SPL; ++r)
                if (EXACT || base + lane + 32 * r < a.up) o[32 * r] = tanhf(__double2float_rn(acc[r]));
        }
    }
}

// Persistent: CTA c owns the frames [c F / G, (c + 1) F / G) of the
// flattened (utterance, frame) sequence (F = B n_mel, G = gridDim.x), in
// chunks of at most frames_per_cta frames within one utterance.  The running
// sums carry from chunk to chunk (a CTA scans its utterance from frame 0 once).
// Prologue: warp w reconstructs harmonics w and w + 8; then all threads build
// the chunk's run tables, one (harmonic, frame) entry each.  Then each warp takes
// whole frames: lane l computes the samples l, l + 32, ... of the frame, all 9
// harmonics (h outer, so the engine's sum over h runs in order in each
// sample's accumulator).
// PRE: the frame starts come from k_nsf_phase_starts, parked in each frame's
// own output samples (9 doubles at out[b][m up ..]); the chunk reads them
// before any of its samples are written, and no other CTA touches them.
template <int SPL, bool EXACT, bool PRE>
__global__ void __launch_bounds__(kNsfThreads, 3) k_nsf_source(NsfArgs a) {
    extern __shared__ double nsf_smem[];
    const int fpc = a.frames_per_cta;
    double* xs = nsf_smem;                                         // [kHarm][fpc]
    FrameRun* tb = reinterpret_cast<FrameRun*>(xs + kHarm * fpc);  // [kHarm][fpc]
    __shared__ float s_lw[kHarm];
    __shared__ double s_pc[2 * kHarm];  // (sin p_h, cos p_h) of this chunk's utterance
    __shared__ int s_next;
    const int w = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t total = a.B * a.n_mel;
    const int64_t g0 = total * blockIdx.x / gridDim.x;
    const int64_t g1 = total * (blockIdx.x + 1) / gridDim.x;
    grid_dep_wait();
    grid_dep_launch();
    if (threadIdx.x < kHarm) s_lw[threadIdx.x] = a.lw[threadIdx.x];
    double x_carry[2] = {0.0, 0.0};  // harmonics w, w + 8: cs at frame carry_m of carry_b
    int64_t carry_m = 0, carry_b = -1;
    for (int64_t g = g0; g < g1;) {
        const int64_t b = g / a.n_mel;
        const int64_t m0 = g - b * a.n_mel;
        int64_t m_end = a.n_mel;
        if (m_end > m0 + fpc) m_end = m0 + fpc;
        if (m_end > g1 - b * a.n_mel) m_end = g1 - b * a.n_mel;
        g = b * a.n_mel + m_end;
        const float* f0b = a.f0 + b * a.n_mel;
        if (b != carry_b) {
            x_carry[0] = x_carry[1] = 0.0;
            carry_m = 0;
            carry_b = b;
        }
        __syncthreads();  // the previous chunk's readers are done with xs / tb / s_next
        if constexpr (PRE) {
            const int nfr = (int)(m_end - m0);
            const double* pre = reinterpret_cast<const double*>(a.out + b * a.T + m0 * a.up);
            const int64_t pstride = a.up / 2;  // doubles per frame of output
            for (int e = threadIdx.x; e < kHarm * nfr; e += kNsfThreads) {
                const int h = e / nfr, mi = e - h * nfr;
                xs[h * fpc + mi] = pre[mi * pstride + h];
            }
        } else {
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int h = w + kNsfWarps * k;
                if (h < kHarm)
                    x_carry[k] = nsf_prologue(a, h, f0b, carry_m, x_carry[k], m0, m_end,
                                              xs + (int64_t)h * fpc);
            }
            carry_m = m_end;
        }
        __syncthreads();  // every harmonic's frame starts are in xs
        // run tables: one (harmonic, frame) entry per thread, all warps sharing
        // the 9 harmonics evenly
        {
            const int nfr = (int)(m_end - m0);
            for (int e = threadIdx.x; e < kHarm * nfr; e += kNsfThreads) {
                const int h = e / nfr, mi = e - h * nfr;
                nsf_frame_entry(a, h, f0b, m0 + mi, xs[h * fpc + mi], tb + h * fpc + mi);
            }
        }
        if (threadIdx.x == 0) s_next = 0;
        if (threadIdx.x < kHarm) {
            const double p =
                threadIdx.x == 0 ? 0.0 : (double)__ldg(a.phase + b * kHarm + threadIdx.x);
            sincos(p, &s_pc[2 * threadIdx.x], &s_pc[2 * threadIdx.x + 1]);
        }
        __syncthreads();
        nsf_frames<SPL, EXACT>(a, b, f0b, m0, m_end, tb, s_lw, s_pc, &s_next, lane);
    }
}

// The exact running sum at every frame start of every (utterance, harmonic),
// one warp each over the whole utterance (the engine's sequence, replayed as
// in nsf_prologue): written as doubles into the first 9 doubles of each
// frame's output samples, out[b][m up + 2 h .. + 1] (up even, up >= 18), for
// k_nsf_source<.., PRE> to read back.  Two warps per CTA spread the B * 9
// serial scans over the SMs.
// With n_mel <= kPreSmemFrames each warp first forms its harmonic's increments
// for the whole utterance in shared memory (the scan's steps then read them
// at shared-memory latency instead of loading f0 and multiplying each step).
constexpr int kPreWarps = 2;
constexpr int kPreSmemFrames = 3072;  // 24 KB per warp
__global__ void __launch_bounds__(32 * kPreWarps) k_nsf_phase_starts(NsfArgs a) {
    extern __shared__ double pre_inc[];  // [kPreWarps][n_mel] when it fits
    grid_dep_wait();
    grid_dep_launch();
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t g = (int64_t)blockIdx.x * kPreWarps + w;
    if (g >= a.B * kHarm) return;
    const int64_t b = g / kHarm;
    const int h = (int)(g - b * kHarm);
    const float* f0b = a.f0 + b * a.n_mel;
    double* inc = nullptr;
    if (a.n_mel <= kPreSmemFrames) {
        inc = pre_inc + (int64_t)w * a.n_mel;
        for (int64_t m = lane; m < a.n_mel; m += 32) inc[m] = increment(__ldg(f0b + m), h, a.inv_sr);
        __syncwarp();
    }
    double* xs = reinterpret_cast<double*>(a.out + b * a.T) + h;
    nsf_prologue(a, h, f0b, 0, 0.0, 0, a.n_mel, xs, a.up / 2, inc);
}

// ------------------------------------------------------------ STFT / iSTFT --

constexpr int kMaxFft = 32;
constexpr int kDspThreads = 256;

// sin and cos of x for |x| <= 1 (the iSTFT applies them to phase = sin(raw)):
// the Taylor series to x^11 / x^10 in f32 Horner form, without the range
// reduction a general sincosf needs.  The first dropped terms are below
// 1/13! = 1.6e-10 and 1/12! = 2.1e-9 on [-1, 1], under 0.07 ulp of the
// results (|sin x| >= 0.84 |x|, cos x >= 0.54 there).
__device__ __forceinline__ void sincos_unit(float x, float* s, float* c) {
    const float x2 = x * x;
    float ps = fmaf(x2, -1.0f / 39916800.0f, 1.0f / 362880.0f);  // x^11, x^9
    ps = fmaf(x2, ps, -1.0f / 5040.0f);                            // x^7
    ps = fmaf(x2, ps, 1.0f / 120.0f);                              // x^5
    ps = fmaf(x2, ps, -1.0f / 6.0f);                               // x^3
    *s = fmaf(x * x2, ps, x);
    float pc = fmaf(x2, -1.0f / 3628800.0f, 1.0f / 40320.0f);      // x^10, x^8
    pc = fmaf(x2, pc, -1.0f / 720.0f);                             // x^6
    pc = fmaf(x2, pc, 1.0f / 24.0f);                               // x^4
    pc = fmaf(x2, pc, -0.5f);                                      // x^2
    *c = fmaf(x2, pc, 1.0f);
}

// cos / sin of 2 pi k n / N (sign of the forward transform applied by the caller)
__device__ __forceinline__ void twiddle(int k, int n, int N, double* c, double* s) {
    sincospi(2.0 * (double)((k * n) % N) / (double)N, s, c);
}

struct StftArgs {
    const float* x;  // [B][T]
    const float* window;
    float* out;
    int64_t B, T, Ts;
    int N, hop, layout, frames_per_cta;
    int64_t tiles_per_b;  // persistent kernels: tiles per utterance
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
    int64_t B, Tf, Ta;
    int N, hop, layout, samples_per_cta;
    float limit;
    int64_t tiles_per_b;  // persistent kernels: tiles per utterance
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
        const float phs = sinf(praw);  // |phs| <= 1
        float sp, cp;
        sincos_unit(phs, &sp, &cp);
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

// ---- power-of-two n_fft (8, 16, 32): one thread per frame, everything static --
//
// Shared layout of both kernels: cos / sin(2 pi j / N) for j < N (double,
// read as broadcasts: every lane of a warp asks for the same j), the window,
// then the kernel's tile.  Output / input rows are staged with a padded
// stride of 2 nb + 1 floats (odd: conflict-free per-thread rows) so global
// memory is read and written in coalesced runs.

template <int N>
constexpr size_t pow2_table_bytes() { return 2 * N * sizeof(double) + kMaxFft * sizeof(float); }

template <int N>
__device__ __forceinline__ void pow2_tables(double* cs, double* sn) {
    for (int j = threadIdx.x; j < N; j += blockDim.x) sincospi(2.0 * j / N, sn + j, cs + j);
}

// STFT: frame f of the tile = thread f.  Real input folds the DFT:
// X_k = x0 + (-1)^k x_{N/2} + sum_{n<N/2} (x_n + x_{N-n}) cos(2 pi k n / N)
//       - i sum_{n<N/2} (x_n - x_{N-n}) sin(2 pi k n / N).
template <int N>
__global__ void __launch_bounds__(kDspThreads) k_stft_pow2(StftArgs a) {
    constexpr int nb = N / 2 + 1, half = N / 2, pad = N / 2, row = 2 * nb + 1;
    extern __shared__ double sm[];
    double* cs = sm;
    double* sn = cs + N;
    float* win = reinterpret_cast<float*>(sn + N);
    float* smp = win + kMaxFft;                                    // [(F-1) hop + N]
    float* os = smp + ((a.frames_per_cta - 1) * a.hop + N + 3) / 4 * 4;  // [F][row]
    const int64_t b = blockIdx.y;
    const int64_t t0 = (int64_t)blockIdx.x * a.frames_per_cta;
    int F = a.frames_per_cta;
    if (t0 + F > a.Ts) F = (int)(a.Ts - t0);
    const int ns = (F - 1) * a.hop + N;
    pow2_tables<N>(cs, sn);
    grid_dep_wait();
    grid_dep_launch();
    const float* xb = a.x + b * a.T;
    for (int i = threadIdx.x; i < N; i += blockDim.x) win[i] = __ldg(a.window + i);
    for (int i = threadIdx.x; i < ns; i += blockDim.x)
        smp[i] = padded_sample(xb, a.T, pad, t0 * a.hop + i);
    __syncthreads();
    for (int f = threadIdx.x; f < F; f += blockDim.x) {
        float fr[N];
#pragma unroll
        for (int n = 0; n < N; ++n) fr[n] = __fmul_rn(smp[f * a.hop + n], win[n]);
        double p[half], q[half];
#pragma unroll
        for (int n = 1; n < half; ++n) {
            p[n] = (double)fr[n] + (double)fr[N - n];
            q[n] = (double)fr[n] - (double)fr[N - n];
        }
        float* o = os + f * row;
#pragma unroll
        for (int k = 0; k < nb; ++k) {
            double re = (double)fr[0] + ((k & 1) ? -(double)fr[half] : (double)fr[half]);
            double im = 0.0;
#pragma unroll
            for (int n = 1; n < half; ++n) {
                re = fma(p[n], cs[(k * n) % N], re);
                im = fma(-q[n], sn[(k * n) % N], im);
            }
            o[k] = __double2float_rn(re);
            o[nb + k] = __double2float_rn(im);
        }
    }
    __syncthreads();
    if (a.layout == CBX_LAYOUT_BTC) {
        float* dst = a.out + (b * a.Ts + t0) * 2 * nb;
        for (int e = threadIdx.x; e < F * 2 * nb; e += blockDim.x)
            dst[e] = os[(e / (2 * nb)) * row + e % (2 * nb)];
    } else {
        for (int c = 0; c < 2 * nb; ++c) {
            float* dst = a.out + (b * 2 * nb + c) * a.Ts + t0;
            for (int f = threadIdx.x; f < F; f += blockDim.x) dst[f] = os[f * row + c];
        }
    }
}

// iSTFT tail: the raw conv_post rows of the tile's frames are staged
// coalesced; thread = frame forms (re, im) in f32 as the engine, then the
// folded inverse DFT in double: for n <= N/2,
//   A = re_0 + (-1)^n re_{N/2} + sum_k 2 re_k cos(2 pi k n / N),
//   S = sum_k 2 im_k sin(2 pi k n / N),  x_n = (A - S) / N, x_{N-n} = (A + S) / N
// (1/N exact for a power of two), windowed into fr[]; then one thread per
// output sample runs the overlap-add in frame order.
template <int N, int HOP>
__global__ void __launch_bounds__(kDspThreads) k_istft_pow2(IstftArgs a) {
    constexpr int nb = N / 2 + 1, half = N / 2, pad = N / 2, row = 2 * nb + 1, frow = N + 1;
    constexpr int kSh = HOP == 1 ? 0 : HOP == 2 ? 1 : HOP == 4 ? 2 : HOP == 8 ? 3 : HOP == 16 ? 4 : 5;
    static_assert((1 << kSh) == HOP, "HOP must be a power of two <= 32");
    extern __shared__ double sm[];
    double* cs = sm;
    double* sn = cs + N;
    float* win = reinterpret_cast<float*>(sn + N);
    const int max_nf = ((a.samples_per_cta + N - 2) >> kSh) + 2;
    float* raw = win + kMaxFft;        // [max_nf][row]
    float* fr = raw + max_nf * row;    // [max_nf][frow]
    const int64_t b = blockIdx.y;
    const int64_t i0 = (int64_t)blockIdx.x * a.samples_per_cta;
    int S = a.samples_per_cta;
    if (i0 + S > a.Ta) S = (int)(a.Ta - i0);
    const int64_t p_lo = i0 + pad, p_hi = i0 + pad + S - 1;
    const int64_t f_lo = p_lo - N + 1 > 0 ? (p_lo - N + 1 + HOP - 1) >> kSh : 0;
    int64_t f_hi = p_hi >> kSh;
    if (f_hi > a.Tf - 1) f_hi = a.Tf - 1;
    const int nf = (int)(f_hi - f_lo + 1);
    pow2_tables<N>(cs, sn);
    grid_dep_wait();
    grid_dep_launch();
    for (int i = threadIdx.x; i < N; i += blockDim.x) win[i] = __ldg(a.window + i);
    if (a.layout == CBX_LAYOUT_BTC) {
        const float* src = a.post + (b * a.Tf + f_lo) * 2 * nb;
        for (int e = threadIdx.x; e < nf * 2 * nb; e += blockDim.x)
            raw[(e / (2 * nb)) * row + e % (2 * nb)] = __ldg(src + e);
    } else {
        for (int c = 0; c < 2 * nb; ++c) {
            const float* src = a.post + (b * 2 * nb + c) * a.Tf + f_lo;
            for (int f = threadIdx.x; f < nf; f += blockDim.x) raw[f * row + c] = __ldg(src + f);
        }
    }
    __syncthreads();
    constexpr double kInvN = 1.0 / N;
    for (int f = threadIdx.x; f < nf; f += blockDim.x) {
        const float* r = raw + f * row;
        float re[nb], im[nb];
#pragma unroll
        for (int k = 0; k < nb; ++k) {
            const float e = expf(r[k]);
            const float mag = (100.0f < e) ? 100.0f : e;  // std::min(exp(raw), 100.0f)
            const float phs = sinf(r[nb + k]);  // |phs| <= 1
            float sp, cp;
            sincos_unit(phs, &sp, &cp);
            re[k] = __fmul_rn(mag, cp);
            im[k] = __fmul_rn(mag, sp);
        }
        const double r0 = (double)re[0], rn = (double)re[nb - 1];
        double re2[nb], im2[nb];
#pragma unroll
        for (int k = 1; k < nb - 1; ++k) {
            re2[k] = 2.0 * (double)re[k];
            im2[k] = 2.0 * (double)im[k];
        }
        float* o = fr + f * frow;
#pragma unroll
        for (int n = 0; n <= half; ++n) {
            double A = r0 + ((n & 1) ? -rn : rn);
            double Sv = 0.0;
#pragma unroll
            for (int k = 1; k < nb - 1; ++k) {
                A = fma(re2[k], cs[(k * n) % N], A);
                Sv = fma(im2[k], sn[(k * n) % N], Sv);
            }
            o[n] = __fmul_rn(__double2float_rn((A - Sv) * kInvN), win[n]);
            if (n != 0 && n != half)
                o[N - n] = __fmul_rn(__double2float_rn((A + Sv) * kInvN), win[N - n]);
        }
    }
    __syncthreads();
    // overlap-add: output sample p (padded position) takes frames t with
    // t HOP <= p <= t HOP + N - 1, in ascending t; q = p - f_lo HOP >= 0
    const int q0 = (int)(i0 + pad - f_lo * HOP);
    for (int i = threadIdx.x; i < S; i += blockDim.x) {
        const int q = q0 + i;
        int tr = q >= N - 1 ? (q - N + 1 + HOP - 1) >> kSh : 0;
        int tr_hi = q >> kSh;
        if (tr_hi > nf - 1) tr_hi = nf - 1;
        float acc = 0.0f, wsum = 0.0f;
        for (; tr <= tr_hi; ++tr) {
            const int n = q - tr * HOP;
            acc = __fadd_rn(acc, fr[tr * frow + n]);
            wsum = __fadd_rn(wsum, __fmul_rn(win[n], win[n]));
        }
        if (wsum > 1e-11f) acc = __fdiv_rn(acc, wsum);
        const float lim = a.limit;
        a.out[b * a.Ta + i0 + i] = (acc < -lim) ? -lim : ((lim < acc) ? lim : acc);
    }
}

// ------------------------------------------ persistent bulk-copy STFT / iSTFT --
// The engine's configuration (n_fft 16, hop 4) and n_fft 8 / hop 2, with
// 16-byte aligned inputs: persistent CTAs loop over (utterance, tile) pairs.
// Each tile's input span arrives in a two-stage shared ring by bulk async
// copies (cp.async.bulk into shared memory, completion counted on an mbarrier
// as transaction bytes), issued two tiles ahead, so loads overlap the
// transforms.  Spans are widened to 16-byte boundaries; only a span that ends
// in the last partial 16 bytes of the whole input gets those few floats by
// plain loads.  The DFT twiddles are compile-time constants (constant-bank
// operands, no shared-memory loads), and the iSTFT's phase sin is sin_cw.

// cos / sin of 2 pi j / 32 from the Taylor series on [0, pi/4] and the octant
// and quadrant symmetries, evaluated by the compiler in double (within an ulp
// of the correctly rounded values).
constexpr double kPiD = 3.14159265358979323846;

constexpr void cx_sincos(double x, double& s, double& c) {  // |x| <= pi / 4
    double ts = x, tc = 1.0;
    s = x;
    c = 1.0;
    for (int i = 1; i < 13; ++i) {
        ts *= -x * x / ((2.0 * i) * (2.0 * i + 1.0));
        tc *= -x * x / ((2.0 * i - 1.0) * (2.0 * i));
        s += ts;
        c += tc;
    }
}

struct DftTable {
    double c[32];
    double s[32];
};

// table[j] = scale * (cos, sin)(2 pi j / N), j < N (N divides 32)
constexpr DftTable make_dft_table(int N, double scale) {
    DftTable t{};
    for (int j = 0; j < N; ++j) {
        const int k = j * (32 / N);  // angle = k pi / 16 = q pi / 2 + r pi / 16
        const int q = k / 8, r = k % 8;
        double s0 = 0.0, c0 = 0.0;
        if (r <= 4) {
            cx_sincos(r * kPiD / 16.0, s0, c0);
        } else {
            cx_sincos((8 - r) * kPiD / 16.0, c0, s0);  // sin(x) = cos(pi/2 - x)
        }
        const double c = q == 0 ? c0 : q == 1 ? -s0 : q == 2 ? -c0 : s0;
        const double s = q == 0 ? s0 : q == 1 ? c0 : q == 2 ? -s0 : -c0;
        t.c[j] = c * scale;
        t.s[j] = s * scale;
    }
    return t;
}

// Forward (STFT): cos, sin.  Inverse (iSTFT): 2 cos / N, 2 sin / N — the
// folded pairs' factor 2 and the 1/N are powers of two, so folding them into
// the table changes no rounding of the sums.
__constant__ DftTable kDft8 = make_dft_table(8, 1.0);
__constant__ DftTable kDft16 = make_dft_table(16, 1.0);
__constant__ DftTable kIdft8 = make_dft_table(8, 2.0 / 8);
__constant__ DftTable kIdft16 = make_dft_table(16, 2.0 / 16);

template <int N>
__device__ __forceinline__ const DftTable& dft_table() {
    static_assert(N == 8 || N == 16, "bulk DSP kernels cover n_fft 8 and 16");
    if constexpr (N == 8) return kDft8;
    else return kDft16;
}
template <int N>
__device__ __forceinline__ const DftTable& idft_table() {
    static_assert(N == 8 || N == 16, "bulk DSP kernels cover n_fft 8 and 16");
    if constexpr (N == 8) return kIdft8;
    else return kIdft16;
}

constexpr int log2_pow2(int v) { return v <= 1 ? 0 : 1 + log2_pow2(v / 2); }

// Span [s, e) of a flat f32 input of E floats (base 16-byte aligned) for a
// bulk copy into `dst`: the copy covers [lo, hi) with lo = s rounded down to
// 4 floats and hi = e rounded up, clipped to the input's last full 16 bytes;
// element g lands at dst[g - lo].  Returns the copy's bytes (0: none) and
// loads the floats in [max(hi, s), e) that the copy cannot reach.
__device__ __forceinline__ uint32_t bulk_span(float* dst, const float* base, int64_t s, int64_t e,
                                              int64_t E, uint64_t* bar) {
    const int64_t lo = s & ~(int64_t)3;
    int64_t hi = (e + 3) & ~(int64_t)3;
    const int64_t e_al = E & ~(int64_t)3;
    if (hi > e_al) hi = e_al;
    uint32_t bytes = 0;
    if (hi > lo) {
        bytes = (uint32_t)((hi - lo) * 4);
        bulk_g2s(dst, base + lo, bytes, bar);
    }
    for (int64_t g = hi > s ? hi : s; g < e; ++g) dst[g - lo] = __ldg(base + g);
    return bytes;
}

template <int N, int HOP, int LAYOUT>
struct IstftTile {
    static constexpr int nb = N / 2 + 1, C2 = 2 * nb, pad = N / 2, frow = N + 1;
    static constexpr int kSh = log2_pow2(HOP);
    static constexpr int kFrames = kDspThreads;  // frames per tile, one per thread
    // output samples per tile: any S consecutive samples need at most
    // (S + N - 2) / HOP + 2 = kFrames frames
    static constexpr int S = (kFrames - 2) * HOP - N + 2;
    static constexpr int RS = (kFrames + 8 + 3) / 4 * 4;  // [C2][RS] row stride (BCT)
    static constexpr int kStage = LAYOUT == CBX_LAYOUT_BTC ? (kFrames * C2 + 8 + 3) / 4 * 4 : C2 * RS;
    static constexpr int kFr = kFrames * frow;
    static constexpr size_t kSmem = (size_t)(2 * kStage + 2 * kFr + N + HOP) * sizeof(float);
    static_assert((1 << kSh) == HOP && HOP <= N && N % HOP == 0, "power-of-two hop <= n_fft");
    static_assert(S > 0, "tile too small");

    int64_t b, i0, f_lo;
    int Sx, nf;
    __device__ __forceinline__ IstftTile(const IstftArgs& a, int64_t tile) {
        b = tile / a.tiles_per_b;
        i0 = (tile - b * a.tiles_per_b) * S;
        Sx = a.Ta - i0 < S ? (int)(a.Ta - i0) : S;
        const int64_t p_lo = i0 + pad, p_hi = i0 + pad + Sx - 1;
        f_lo = p_lo - N + 1 > 0 ? (p_lo - N + 1 + HOP - 1) >> kSh : 0;
        int64_t f_hi = p_hi >> kSh;
        if (f_hi > a.Tf - 1) f_hi = a.Tf - 1;
        nf = (int)(f_hi - f_lo + 1);
    }
    // thread 0: bulk copies of the tile's conv_post frames into `dst`
    __device__ __forceinline__ void issue(const IstftArgs& a, float* dst, uint64_t* bar) const {
        const int64_t E = a.B * a.Tf * C2;
        uint32_t bytes = 0;
        if constexpr (LAYOUT == CBX_LAYOUT_BTC) {
            const int64_t s = (b * a.Tf + f_lo) * C2;
            // expect the bytes first: complete_tx must not precede expect_tx
            const int64_t lo = s & ~(int64_t)3;
            int64_t hi = (s + (int64_t)nf * C2 + 3) & ~(int64_t)3;
            if (hi > (E & ~(int64_t)3)) hi = E & ~(int64_t)3;
            if (hi > lo) mbar_arrive_expect_tx(bar, (uint32_t)((hi - lo) * 4));
            bytes = bulk_span(dst, a.post, s, s + (int64_t)nf * C2, E, bar);
        } else {
            uint32_t total = 0;
            for (int c = 0; c < C2; ++c) {
                const int64_t s = (b * C2 + c) * a.Tf + f_lo;
                const int64_t lo = s & ~(int64_t)3;
                int64_t hi = (s + nf + 3) & ~(int64_t)3;
                if (hi > (E & ~(int64_t)3)) hi = E & ~(int64_t)3;
                if (hi > lo) total += (uint32_t)((hi - lo) * 4);
            }
            if (total) mbar_arrive_expect_tx(bar, total);
            for (int c = 0; c < C2; ++c) {
                const int64_t s = (b * C2 + c) * a.Tf + f_lo;
                bytes += bulk_span(dst + c * RS, a.post, s, s + nf, E, bar);
            }
        }
        if (bytes == 0) mbar_arrive(bar);  // nothing in flight: complete the phase now
    }
};

template <int N, int HOP, int LAYOUT>
__global__ void __launch_bounds__(kDspThreads, 3) k_istft_bulk(IstftArgs a, int* dev_err) {
    using G = IstftTile<N, HOP, LAYOUT>;
    constexpr int nb = G::nb, C2 = G::C2, half = N / 2, pad = G::pad, frow = G::frow;
    constexpr int NH = N / HOP;
    extern __shared__ __align__(16) float smf[];
    __shared__ uint64_t bars[2];
    float* raw0 = smf;                    // [2][kStage]
    float* fr0 = smf + 2 * G::kStage;     // [2][kFrames][frow]
    float* win = fr0 + 2 * G::kFr;        // [N]
    float* wsq = win + N;                 // [HOP]
    const int64_t n_tiles = a.B * a.tiles_per_b;
    const int64_t mine =
        n_tiles > (int64_t)blockIdx.x ? (n_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    if (threadIdx.x == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        mbar_fence_init();
    }
    grid_dep_wait();
    grid_dep_launch();
    if (threadIdx.x == 0)
        for (int64_t k = 0; k < mine && k < 2; ++k)
            G(a, blockIdx.x + k * gridDim.x).issue(a, raw0 + k * G::kStage, &bars[k]);
    if (threadIdx.x < N) win[threadIdx.x] = __ldg(a.window + threadIdx.x);
    // orders the mbarrier inits (polled below) and the window
    __syncthreads();
    if (threadIdx.x < HOP) {
        // an interior sample's window-square sum, frames in ascending order
        // (window index descending), as the engine accumulates it
        float w = 0.0f;
#pragma unroll
        for (int m = NH - 1; m >= 0; --m) {
            const float v = win[threadIdx.x + m * HOP];
            w = __fadd_rn(w, __fmul_rn(v, v));
        }
        wsq[threadIdx.x] = w;
    }
    const DftTable& tw = idft_table<N>();
    const float lim = a.limit;
    for (int64_t k = 0; k < mine; ++k) {
        const int64_t tile = blockIdx.x + k * gridDim.x;
        const int st = (int)(k & 1);
        const G g(a, tile);
        const bool ok = mbar_wait_bounded(&bars[st], (uint32_t)((k >> 1) & 1));
        const float* raw = raw0 + st * G::kStage;
        float* fr = fr0 + st * G::kFr;
        const int f = threadIdx.x;
        if (f < g.nf) {
            float v[C2];
            if constexpr (LAYOUT == CBX_LAYOUT_BTC) {
                // the span starts at an even float (C2 is even): 8-byte loads
                const int off = (int)(((g.b * a.Tf + g.f_lo) * C2) & 3);
                const float2* rp = reinterpret_cast<const float2*>(raw + off + f * C2);
#pragma unroll
                for (int j = 0; j < C2 / 2; ++j) {
                    const float2 t = rp[j];
                    v[2 * j] = t.x;
                    v[2 * j + 1] = t.y;
                }
            } else {
                const int64_t s0 = g.b * C2 * a.Tf + g.f_lo;
                const int o0 = (int)(s0 & 3), step = (int)(a.Tf & 3);
#pragma unroll
                for (int c = 0; c < C2; ++c) v[c] = raw[c * G::RS + ((o0 + c * step) & 3) + f];
            }
            // magnitude / phase -> (re, im) in f32 as hift_vocoder.cpp:795-803
            double rd[nb], id[nb];
#pragma unroll
            for (int q = 0; q < nb; ++q) {
                const float e = expf(v[q]);
                const float mag = (100.0f < e) ? 100.0f : e;  // std::min(exp(raw), 100.0f)
                const float phs = sin_cw(v[nb + q]);          // |phs| <= 1
                float sp, cp;
                sincos_unit(phs, &sp, &cp);
                rd[q] = (double)__fmul_rn(mag, cp);
                id[q] = (double)__fmul_rn(mag, sp);
            }
            // folded inverse DFT in double, 1/N and the factor 2 in the table
            constexpr double kInvN = 1.0 / N;
            const double r0 = rd[0] * kInvN, rn = rd[nb - 1] * kInvN;
            float* o = fr + f * frow;
            // positions n and m = half - n share the even-k and odd-k partial
            // sums: c(k m) = (-1)^k c(k n), s(k m) = -(-1)^k s(k n) (~40% fewer
            // FP64 operations); x_n = A_n - S_n, x_{N-n} = A_n + S_n
#pragma unroll
            for (int n = 0; n <= half / 2; ++n) {
                const double B = r0 + ((n & 1) ? -rn : rn);  // also for m (half even)
                double Ek = 0.0, Ok = 0.0, Es = 0.0, Os = 0.0;
#pragma unroll
                for (int q = 1; q < nb - 1; ++q) {
                    const double c = tw.c[(q * n) % N], sv = tw.s[(q * n) % N];
                    if (q & 1) {
                        Ok = fma(rd[q], c, Ok);
                        Os = fma(id[q], sv, Os);
                    } else {
                        Ek = fma(rd[q], c, Ek);
                        Es = fma(id[q], sv, Es);
                    }
                }
                const double BE = B + Ek;
                const double An = BE + Ok, Sn = Es + Os;
                o[n] = __fmul_rn(__double2float_rn(An - Sn), win[n]);
                if (n != 0) o[N - n] = __fmul_rn(__double2float_rn(An + Sn), win[N - n]);
                const int m = half - n;
                if (m != n) {
                    const double Am = BE - Ok, Sm = Os - Es;
                    o[m] = __fmul_rn(__double2float_rn(Am - Sm), win[m]);
                    if (m != half) o[N - m] = __fmul_rn(__double2float_rn(Am + Sm), win[N - m]);
                }
            }
        }
        // frames complete and this stage's raw span consumed; a failed wait
        // anywhere makes the whole CTA leave together
        if (__syncthreads_or(ok ? 0 : 1)) {
            if (threadIdx.x == 0) {
                if (dev_err) atomicOr(dev_err, CBX_DEVERR_WAIT_TIMEOUT);
                if (k + 1 < mine) mbar_wait_bounded(&bars[st ^ 1], (uint32_t)(((k + 1) >> 1) & 1));
            }
            return;
        }
        if (threadIdx.x == 0 && k + 2 < mine)
            G(a, tile + 2 * (int64_t)gridDim.x).issue(a, raw0 + st * G::kStage, &bars[st]);
        // overlap-add in ascending frame order, window-square division, clamp
        const int q0 = (int)(g.i0 + pad - g.f_lo * HOP);
        float* outp = a.out + g.b * a.Ta + g.i0;
        const int64_t p_end = a.Tf * HOP;
        // every sample of the tile has its full NH frames (no edge samples)
        const bool all_interior = g.i0 + pad >= N - HOP && g.i0 + pad + g.Sx <= p_end;
        for (int i = threadIdx.x; i < g.Sx; i += kDspThreads) {
            const int q = q0 + i;
            const int64_t p = g.i0 + pad + i;
            float acc = 0.0f, wsum;
            if (all_interior || (p >= N - HOP && p < p_end)) {  // NH frames: t = trh - NH + 1 .. trh
                const int j = q & (HOP - 1), trh = q >> G::kSh;
#pragma unroll
                for (int m = NH - 1; m >= 0; --m)
                    acc = __fadd_rn(acc, fr[(trh - m) * frow + j + m * HOP]);
                wsum = wsq[j];
            } else {
                wsum = 0.0f;
                int tr = q >= N - 1 ? (q - N + 1 + HOP - 1) >> G::kSh : 0;
                int tr_hi = q >> G::kSh;
                if (tr_hi > g.nf - 1) tr_hi = g.nf - 1;
                for (; tr <= tr_hi; ++tr) {
                    const int n = q - tr * HOP;
                    acc = __fadd_rn(acc, fr[tr * frow + n]);
                    wsum = __fadd_rn(wsum, __fmul_rn(win[n], win[n]));
                }
            }
            if (wsum > 1e-11f) acc = __fdiv_rn(acc, wsum);
            outp[i] = (acc < -lim) ? -lim : ((lim < acc) ? lim : acc);
        }
    }
}

template <int N, int HOP, int LAYOUT>
struct StftTile {
    static constexpr int nb = N / 2 + 1, C2 = 2 * nb, pad = N / 2, half = N / 2;
    static constexpr int kFrames = kDspThreads;  // frames per tile, one per thread
    static constexpr int kSpan = (kFrames - 1) * HOP + N;  // padded samples per tile
    static constexpr int kStage = (kSpan + 8 + 3) / 4 * 4;
    static constexpr int row = C2 + 1;  // odd: conflict-free per-thread rows
    static constexpr int kOut = kFrames * row;
    static constexpr size_t kSmem = (size_t)(2 * kStage + 2 * kOut + N) * sizeof(float);
    static_assert(HOP <= N, "hop <= n_fft");

    int64_t b, t0;
    int F;
    int64_t a_lo, a_hi;  // audio samples [a_lo, a_hi) of the tile's padded span
    __device__ __forceinline__ StftTile(const StftArgs& a, int64_t tile) {
        b = tile / a.tiles_per_b;
        t0 = (tile - b * a.tiles_per_b) * kFrames;
        F = a.Ts - t0 < kFrames ? (int)(a.Ts - t0) : kFrames;
        const int64_t ax0 = t0 * HOP - pad;
        a_lo = ax0 < 0 ? 0 : ax0;
        a_hi = ax0 + (int64_t)(F - 1) * HOP + N;
        if (a_hi > a.T) a_hi = a.T;
    }
    __device__ __forceinline__ int64_t ax0() const { return t0 * HOP - pad; }
    __device__ __forceinline__ bool edge(const StftArgs& a) const {
        return ax0() < 0 || ax0() + (int64_t)(F - 1) * HOP + N > a.T;
    }
    __device__ __forceinline__ void issue(const StftArgs& a, float* dst, uint64_t* bar) const {
        const int64_t E = a.B * a.T;
        const int64_t s = b * a.T + a_lo, e = b * a.T + a_hi;
        const int64_t lo = s & ~(int64_t)3;
        int64_t hi = (e + 3) & ~(int64_t)3;
        if (hi > (E & ~(int64_t)3)) hi = E & ~(int64_t)3;
        if (hi > lo) mbar_arrive_expect_tx(bar, (uint32_t)((hi - lo) * 4));
        if (bulk_span(dst, a.x, s, e, E, bar) == 0) mbar_arrive(bar);
    }
};

// frame[n] = x[n + S] * window[n] (f32, the engine's frame[n] = src[n] * window[n])
template <int N, int S>
__device__ __forceinline__ void window_from(const float (&v)[N + 4], const float* win,
                                            float (&fr)[N]) {
#pragma unroll
    for (int n = 0; n < N; ++n) fr[n] = __fmul_rn(v[n + S], win[n]);
}

template <int N, int HOP, int LAYOUT>
__global__ void __launch_bounds__(kDspThreads, 4) k_stft_bulk(StftArgs a, int* dev_err) {
    using G = StftTile<N, HOP, LAYOUT>;
    constexpr int nb = G::nb, C2 = G::C2, half = G::half, row = G::row;
    extern __shared__ __align__(16) float smf[];
    __shared__ uint64_t bars[2];
    float* smp0 = smf;                  // [2][kStage]
    float* os0 = smf + 2 * G::kStage;   // [2][kFrames][row]
    float* win = os0 + 2 * G::kOut;     // [N]
    const int64_t n_tiles = a.B * a.tiles_per_b;
    const int64_t mine =
        n_tiles > (int64_t)blockIdx.x ? (n_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    if (threadIdx.x == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        mbar_fence_init();
    }
    grid_dep_wait();
    grid_dep_launch();
    if (threadIdx.x == 0)
        for (int64_t k = 0; k < mine && k < 2; ++k)
            G(a, blockIdx.x + k * gridDim.x).issue(a, smp0 + k * G::kStage, &bars[k]);
    if (threadIdx.x < N) win[threadIdx.x] = __ldg(a.window + threadIdx.x);
    __syncthreads();
    const DftTable& tw = dft_table<N>();
    for (int64_t k = 0; k < mine; ++k) {
        const int64_t tile = blockIdx.x + k * gridDim.x;
        const int st = (int)(k & 1);
        const G g(a, tile);
        const bool ok = mbar_wait_bounded(&bars[st], (uint32_t)((k >> 1) & 1));
        const float* smp = smp0 + st * G::kStage;
        float* os = os0 + st * G::kOut;
        // smp[j] holds audio sample (b T + a_lo) rounded down to 4 floats, + j
        const int64_t lo = (g.b * a.T + g.a_lo) & ~(int64_t)3;
        const int64_t base_j = g.b * a.T + g.ax0() - lo;  // smp index of padded sample 0
        const int f = threadIdx.x;
        if (f < g.F) {
            float fr[N];
            if (!g.edge(a)) {
                if constexpr (HOP % 4 == 0) {
                    // the frame's samples start base_j (0..3, uniform per
                    // tile) past a 16-byte boundary: five conflict-free
                    // 16-byte loads cover them, then a compile-time shift
                    float v[N + 4];
                    const float4* s4 = reinterpret_cast<const float4*>(smp + f * HOP);
#pragma unroll
                    for (int c = 0; c < N / 4 + 1; ++c) {
                        const float4 t = s4[c];
                        v[4 * c] = t.x;
                        v[4 * c + 1] = t.y;
                        v[4 * c + 2] = t.z;
                        v[4 * c + 3] = t.w;
                    }
                    switch ((int)base_j) {
                        case 0: window_from<N, 0>(v, win, fr); break;
                        case 1: window_from<N, 1>(v, win, fr); break;
                        case 2: window_from<N, 2>(v, win, fr); break;
                        default: window_from<N, 3>(v, win, fr); break;
                    }
                } else {
                    const float* src = smp + base_j + f * HOP;
#pragma unroll
                    for (int n = 0; n < N; ++n) fr[n] = __fmul_rn(src[n], win[n]);
                }
            } else {
                // reflect padding about the edge samples (hift_vocoder.cpp:473-476)
#pragma unroll
                for (int n = 0; n < N; ++n) {
                    int64_t ai = g.ax0() + (int64_t)f * HOP + n;
                    if (ai < 0) ai = -ai;
                    if (ai >= a.T) ai = 2 * a.T - 2 - ai;
                    const float x = (ai >= g.a_lo && ai < g.a_hi)
                                        ? smp[g.b * a.T + ai - lo]
                                        : __ldg(a.x + g.b * a.T + ai);
                    fr[n] = __fmul_rn(x, win[n]);
                }
            }
            // folded real DFT in double (X_k = sum x_n e^{-2 pi i k n / N})
            double p[half], q[half];
#pragma unroll
            for (int n = 1; n < half; ++n) {
                p[n] = (double)fr[n] + (double)fr[N - n];
                q[n] = (double)fr[n] - (double)fr[N - n];
            }
            const double x0 = (double)fr[0], xh = (double)fr[half];
            float* o = os + f * row;
            // bins k and half - k share the even-n and odd-n partial sums:
            // c((half - k) n) = (-1)^n c(k n), s((half - k) n) = -(-1)^n s(k n),
            // so one pass over n gives both (~40% fewer FP64 operations).  The
            // sine sums accumulate -q s from +0, as the direct sum does, so a
            // bin with no sine content keeps im = +0.
#pragma unroll
            for (int kk = 0; kk <= half / 2; ++kk) {
                const double A = x0 + ((kk & 1) ? -xh : xh);  // also bin half - kk (half even)
                double E = 0.0, O = 0.0, NE = 0.0, NO = 0.0;
#pragma unroll
                for (int n = 1; n < half; ++n) {
                    const double c = tw.c[(kk * n) % N], sv = tw.s[(kk * n) % N];
                    if (n & 1) {
                        O = fma(p[n], c, O);
                        NO = fma(-q[n], sv, NO);
                    } else {
                        E = fma(p[n], c, E);
                        NE = fma(-q[n], sv, NE);
                    }
                }
                const double AE = A + E;
                o[kk] = __double2float_rn(AE + O);
                o[nb + kk] = __double2float_rn(NE + NO);
                if (kk != half - kk) {
                    o[half - kk] = __double2float_rn(AE - O);
                    o[nb + half - kk] = __double2float_rn(NO - NE);
                }
            }
        }
        if (__syncthreads_or(ok ? 0 : 1)) {
            if (threadIdx.x == 0) {
                if (dev_err) atomicOr(dev_err, CBX_DEVERR_WAIT_TIMEOUT);
                if (k + 1 < mine) mbar_wait_bounded(&bars[st ^ 1], (uint32_t)(((k + 1) >> 1) & 1));
            }
            return;
        }
        if (threadIdx.x == 0 && k + 2 < mine)
            G(a, tile + 2 * (int64_t)gridDim.x).issue(a, smp0 + st * G::kStage, &bars[st]);
        // coalesced stores of the staged spectra
        if constexpr (LAYOUT == CBX_LAYOUT_BTC) {
            float* dst = a.out + (g.b * a.Ts + g.t0) * C2;
            for (int e = threadIdx.x; e < g.F * C2; e += kDspThreads) {
                const int fi = e / C2;
                dst[e] = os[fi * row + (e - fi * C2)];
            }
        } else {
#pragma unroll 2
            for (int c = 0; c < C2; ++c) {
                float* dst = a.out + (g.b * C2 + c) * a.Ts + g.t0;
                if (threadIdx.x < g.F) dst[threadIdx.x] = os[threadIdx.x * row + c];
            }
        }
    }
}

// CBX_DSP_TILED=1 selects the one-tile-per-CTA kernels even where the
// persistent bulk-copy kernels apply (A/B comparisons; both are tested).
bool dsp_tiled_only() {
    static const bool v = [] {
        const char* e = getenv("CBX_DSP_TILED");
        return e && e[0] && e[0] != '0';
    }();
    return v;
}

// Persistent launch: as many CTAs per SM as fit (at most the tile count),
// lowered while that leaves the per-CTA tile counts more than 10% uneven.
template <typename K>
int persistent_ctas(K kern, size_t smem, int64_t n_tiles) {
    const int occ = occupancy(kern, kDspThreads, smem);
    const int sms = num_sms();
    int per_sm = occ;
    for (int c = occ; c >= 1; --c) {
        const double avg = (double)n_tiles / ((double)sms * c);
        per_sm = c;
        if (avg >= ceil(avg) * 0.9) break;
    }
    int64_t ctas = (int64_t)sms * per_sm;
    if (ctas > n_tiles) ctas = n_tiles;
    return (int)(ctas < 1 ? 1 : ctas);
}

template <int N, int HOP, int LAYOUT>
int launch_istft_bulk(IstftArgs a, cudaStream_t st) {
    using G = IstftTile<N, HOP, LAYOUT>;
    auto kern = k_istft_bulk<N, HOP, LAYOUT>;
    if (!smem_opt_in(kern, G::kSmem))
        return fail(CBX_ERR_CUDA, "cbx_istft_post: shared memory opt-in failed");
    a.samples_per_cta = G::S;
    a.tiles_per_b = (a.Ta + G::S - 1) / G::S;
    const int ctas = persistent_ctas(kern, G::kSmem, a.B * a.tiles_per_b);
    return launch_status(launch(kern, dim3((unsigned)ctas), dim3(kDspThreads), G::kSmem, st, a,
                                device_error_word()),
                         "cbx_istft_post");
}

template <int N, int HOP, int LAYOUT>
int launch_stft_bulk(StftArgs a, cudaStream_t st) {
    using G = StftTile<N, HOP, LAYOUT>;
    auto kern = k_stft_bulk<N, HOP, LAYOUT>;
    if (!smem_opt_in(kern, G::kSmem))
        return fail(CBX_ERR_CUDA, "cbx_stft: shared memory opt-in failed");
    a.frames_per_cta = G::kFrames;
    a.tiles_per_b = (a.Ts + G::kFrames - 1) / G::kFrames;
    const int ctas = persistent_ctas(kern, G::kSmem, a.B * a.tiles_per_b);
    return launch_status(launch(kern, dim3((unsigned)ctas), dim3(kDspThreads), G::kSmem, st, a,
                                device_error_word()),
                         "cbx_stft");
}

template <int N>
int launch_stft_pow2(StftArgs a, cudaStream_t st) {
    auto bytes = [&](int F) {
        return pow2_table_bytes<N>() + (size_t)(((F - 1) * a.hop + N + 3) / 4 * 4) * 4 +
               (size_t)F * (2 * (N / 2 + 1) + 1) * 4;
    };
    int F = kDspThreads;
    while (F > 32 && bytes(F) > 48 * 1024) F /= 2;
    a.frames_per_cta = F;
    const int64_t tiles = (a.Ts + F - 1) / F;
    return launch_status(launch(k_stft_pow2<N>, dim3((unsigned)tiles, (unsigned)a.B),
                                dim3(kDspThreads), bytes(F), st, a),
                         "cbx_stft");
}

template <int N, int HOP>
int launch_istft_pow2(IstftArgs a, cudaStream_t st) {
    constexpr int nb = N / 2 + 1;
    auto bytes = [&](int S) {
        const int max_nf = (S + N - 2) / a.hop + 2;
        return pow2_table_bytes<N>() + (size_t)max_nf * ((2 * nb + 1) + (N + 1)) * 4;
    };
    // the tile's frames ((S + N - 2) / hop + 2 at most) fit the block, one
    // frame per thread, and the staging fits the default 48 KB
    int S = (kDspThreads - 2) * a.hop - N + 2;
    while (S > 64 && bytes(S) > 48 * 1024) S /= 2;
    a.samples_per_cta = S;
    const int64_t tiles = (a.Ta + S - 1) / S;
    return launch_status(launch(k_istft_pow2<N, HOP>, dim3((unsigned)tiles, (unsigned)a.B),
                                dim3(kDspThreads), bytes(S), st, a),
                         "cbx_istft_post");
}

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
    a.B = B;
    // one wave of persistent CTAs, equal shares of the B * n_mel frames; each
    // CTA keeps a chunk of up to 64 frames' running sums and run tables in
    // shared memory
    const int64_t frames = B * n_mel;
    const int fpc = 64;  // 9 * 64 * (8 + 104) B = 63 KB of frame tables: 3 CTAs per SM
    a.frames_per_cta = fpc;
    const size_t smem = (size_t)kHarm * fpc * (sizeof(double) + sizeof(FrameRun));
    // Frame starts: precomputed once per (utterance, harmonic) by
    // k_nsf_phase_starts and parked in the frames' own output samples when
    // 9 doubles fit there (upsample even, >= 18, output 8-byte aligned);
    // otherwise each CTA replays its utterance up to its frames itself.
    const bool pre = upsample % 2 == 0 && upsample >= 2 * kHarm &&
                     (reinterpret_cast<uintptr_t>(out) & 7u) == 0;
    // the engine's upsample (480 = 32 x 15): one pass of 15 samples per lane
    // with no bounds checks; any other: passes of 16 per lane
    auto kern = upsample == 480 ? (pre ? k_nsf_source<15, true, true> : k_nsf_source<15, true, false>)
                                : (pre ? k_nsf_source<16, false, true> : k_nsf_source<16, false, false>);
    if (!smem_opt_in(kern, smem))
        return fail(CBX_ERR_CUDA, "cbx_nsf_source: shared memory opt-in failed");
    int64_t ctas = (int64_t)num_sms() * occupancy(kern, kNsfThreads, smem);
    if (ctas > (frames + kHarm - 1) / kHarm) ctas = (frames + kHarm - 1) / kHarm;
    if (ctas < 1) ctas = 1;
    if (pre) {
        const int64_t scans = B * kHarm;
        const size_t pre_smem =
            n_mel <= kPreSmemFrames ? (size_t)kPreWarps * n_mel * sizeof(double) : 0;
        if (pre_smem > 48 * 1024 && !smem_opt_in(k_nsf_phase_starts, pre_smem))
            return fail(CBX_ERR_CUDA, "cbx_nsf_source: shared memory opt-in failed");
        const int e = launch_status(launch(k_nsf_phase_starts,
                                           dim3((unsigned)((scans + kPreWarps - 1) / kPreWarps)),
                                           dim3(32 * kPreWarps), pre_smem, stream, a),
                                    "cbx_nsf_source");
        if (e != CBX_OK) return e;
    }
    return launch_status(launch(kern, dim3((unsigned)ctas), dim3(kNsfThreads), smem, stream, a),
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
    a.B = B;
    a.T = T;
    a.Ts = 1 + T / hop;  // 1 + (T + 2 pad - n_fft) / hop with pad = n_fft / 2
    a.N = n_fft;
    a.hop = hop;
    a.layout = layout;
    if (aligned16(audio) && !dsp_tiled_only()) {  // persistent bulk-copy kernels
#define CBX_STFT_BULK(NN, HH)                                                              \
    if (n_fft == NN && hop == HH)                                                          \
        return layout == CBX_LAYOUT_BTC ? launch_stft_bulk<NN, HH, CBX_LAYOUT_BTC>(a, stream) \
                                        : launch_stft_bulk<NN, HH, CBX_LAYOUT_BCT>(a, stream);
        CBX_STFT_BULK(16, 4) CBX_STFT_BULK(8, 2)
#undef CBX_STFT_BULK
    }
    switch (n_fft) {  // power-of-two sizes: thread-per-frame kernels
        case 8: return launch_stft_pow2<8>(a, stream);
        case 16: return launch_stft_pow2<16>(a, stream);
        case 32: return launch_stft_pow2<32>(a, stream);
        default: break;
    }
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
    a.B = B;
    a.Tf = n_frames;
    a.Ta = (n_frames - 1) * hop;
    a.N = n_fft;
    a.hop = hop;
    a.layout = layout;
    a.limit = audio_limit;
    if (aligned16(post) && !dsp_tiled_only()) {  // persistent bulk-copy kernels
#define CBX_ISTFT_BULK(NN, HH)                                                               \
    if (n_fft == NN && hop == HH)                                                            \
        return layout == CBX_LAYOUT_BTC ? launch_istft_bulk<NN, HH, CBX_LAYOUT_BTC>(a, stream) \
                                        : launch_istft_bulk<NN, HH, CBX_LAYOUT_BCT>(a, stream);
        CBX_ISTFT_BULK(16, 4) CBX_ISTFT_BULK(8, 2)
#undef CBX_ISTFT_BULK
    }
    // power-of-two n_fft and hop: one thread per frame, shifts instead of divisions
#define CBX_ISTFT_CASE(NN, HH) \
    if (n_fft == NN && hop == HH) return launch_istft_pow2<NN, HH>(a, stream);
    CBX_ISTFT_CASE(8, 1) CBX_ISTFT_CASE(8, 2) CBX_ISTFT_CASE(8, 4) CBX_ISTFT_CASE(8, 8)
    CBX_ISTFT_CASE(16, 1) CBX_ISTFT_CASE(16, 2) CBX_ISTFT_CASE(16, 4) CBX_ISTFT_CASE(16, 8)
    CBX_ISTFT_CASE(16, 16)
    CBX_ISTFT_CASE(32, 1) CBX_ISTFT_CASE(32, 2) CBX_ISTFT_CASE(32, 4) CBX_ISTFT_CASE(32, 8)
    CBX_ISTFT_CASE(32, 16) CBX_ISTFT_CASE(32, 32)
#undef CBX_ISTFT_CASE
    // other even sizes: one thread per (frame, bin) / (frame, n-pair);
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
