// Register-resident Stockham kernels for batched power-of-two lines (the BASELINE
// config 1/2 hot path, the higher axes of the 3D and 2D-convolution configs, and the
// FullComplex real transforms).
//
// A line of N points is owned by TT = N / E threads, each holding E points in
// registers.  With the load pattern "thread t holds positions t + m*TT", the first
// radix stage's butterflies are formed entirely from the thread's own registers and
// the last stage's outputs land on positions t + m*TT again, so global memory is read
// and written exactly once.  Only the middle stages exchange through one padded
// shared-memory buffer (odd line stride, one pad slot per 16 points: conflict-free).
//
// Layouts: contiguous lines put the TT threads of a line next to each other (a warp
// touches 32 consecutive complex values); strided lines (STRIDED) put the G lines of a
// CTA next to each other instead, so a warp touches G neighbouring lines of the same
// position -- the coalesced access of an ND higher axis without any transpose pass.
//
// Twiddles come from per-stage transposed tables read through the read-only cache.
// Inverse transforms conjugate on load and store (tables stay forward).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "dft_codelets.cuh"
#include "reg_kernels.hpp"

namespace b200fft {

namespace regk {

template <typename T> struct vec2;
template <> struct vec2<float> { using type = float2; };
template <> struct vec2<double> { using type = double2; };

// Shared-memory slot of line position e: one spare slot every 16 positions for
// power-of-two lines (their radix-16 strides would otherwise collapse onto few banks);
// odd-radix lines are unpadded (their stage strides are odd multiples already).
template <int N> __device__ __forceinline__ int pad(int e) { return (N & (N - 1)) == 0 ? e + (e >> 4) : e; }

// Shared-memory stride between the G lines of a CTA (complex elements, >= pad(N-1) + 1).
// A 128-byte wavefront holds W complex values (16 for f32, 8 for f64).  Within one
// wavefront a warp touches L lines at D consecutive positions each: strided layouts put
// the lines fastest (L = min(G, W), D = W / L), contiguous ones the positions (D = min(TT,
// W), L = W / D).  Line g's slot for position t is g*LS + t (+ the same pad), so the
// wavefront is conflict-free when LS = D (mod W): the lines then start D slots apart and
// their D positions fill the gaps.  (LS = N + N/16 + 1 = 1 (mod W) made a strided
// 8-line CTA 2-way conflicted.)
template <typename T>
__host__ __device__ constexpr int reg_ls(int N, int E, int G, bool strided) {
    const int W = sizeof(T) == 4 ? 16 : 8;
    const int TT = N / E;
    int ls = N + N / 16 + 1;
    if (!strided && TT >= W) return ls;  // a wavefront stays inside one line
    const int D = strided ? (G >= W ? 1 : W / G) : TT;
    while (ls % W != D % W) ls++;
    return ls;
}

template <typename T> __device__ __forceinline__ cplx<T> mul(cplx<T> a, cplx<T> b) {
    return {a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x};
}
template <typename T> __device__ __forceinline__ cplx<T> tw_load(const cplx<T> *tw, int64_t idx) {
    auto v = __ldg(reinterpret_cast<const typename vec2<T>::type *>(tw) + idx);
    return {v.x, v.y};
}
template <typename T> __device__ __forceinline__ cplx<T> ld_c(const void *base, int64_t idx) {
    const auto w = __ldcs(reinterpret_cast<const typename vec2<T>::type *>(base) + idx);
    return {w.x, w.y};
}
template <typename T> __device__ __forceinline__ void st_c(void *base, int64_t idx, cplx<T> v) {
    typename vec2<T>::type w;
    w.x = v.x;
    w.y = v.y;
    __stcs(reinterpret_cast<typename vec2<T>::type *>(base) + idx, w);
}

struct LineIO {
    int64_t in_base, out_base;
    bool valid;
    int64_t in_pos0 = 0, out_pos0 = 0;  // Bluestein modes: i * is of each side (block position base)
};

// REG_R2R pre-processing (r2r_ir.rs:1282-1385): the values at the thread's FFT
// positions p = t + m TT of the line's reduction, read from the real line through
// `at(j)` (global memory, or the persistent variant's shared-memory copy).  Type I: even
// / odd extension of length L = 2(n-1) / 2(n+1); II: even-odd reorder (odd sources
// negated for DST); III: (a - i b) A[p] with a, b = x[p], x[n-p] (DST: x[n-1-p],
// x[p-1]); IV with n even: (x[2p] -+ i x[n-1-2p]) A[p]; IV with n odd: x[p] A[p], zero
// for p >= n.  tw2 = [A | B] indexed by FFT position (lower.cpp table_r2r).  The kind
// is uniform, so the switch sits outside the unrolled point loops.
template <typename T, int N, int E, typename At>
__device__ __forceinline__ void r2r_load_all(const RegParams &rp, At at, int t, cplx<T> (&v)[E]) {
    constexpr int TT = N / E;
    const int n = rp.r2r_n;
    const bool dst = rp.r2r_kind >= 4;
    const cplx<T> *A = reinterpret_cast<const cplx<T> *>(rp.tw2);
    switch (rp.r2r_kind & 3) {
        case 0:
#pragma unroll
            for (int m = 0; m < E; m++) {
                const int p = t + m * TT;
                T x = T(0);
                if (!dst)
                    x = at(p < n ? p : N - p);
                else if (p != 0 && p != n + 1)
                    x = p <= n ? at(p - 1) : -at(N - p - 1);
                v[m] = {x, T(0)};
            }
            break;
        case 1: {
            const int split = (n + 1) / 2;
#pragma unroll
            for (int m = 0; m < E; m++) {
                const int p = t + m * TT;
                const int s = p < split ? 2 * p : 2 * (n - p) - 1;
                const T x = at(s);
                v[m] = {(dst && (s & 1)) ? -x : x, T(0)};
            }
            break;
        }
        case 2:
#pragma unroll
            for (int m = 0; m < E; m++) {
                const int p = t + m * TT;
                const T a = dst ? at(n - 1 - p) : at(p);
                const T b = p == 0 ? T(0) : (dst ? at(p - 1) : at(n - p));
                v[m] = mul(cplx<T>{a, -b}, tw_load(A, p));
            }
            break;
        default:
            if ((n & 1) == 0) {
#pragma unroll
                for (int m = 0; m < E; m++) {
                    const int p = t + m * TT;
                    const T a = at(2 * p), b = at(n - 1 - 2 * p);
                    v[m] = mul(cplx<T>{a, dst ? b : -b}, tw_load(A, p));
                }
            } else {
#pragma unroll
                for (int m = 0; m < E; m++) {
                    const int p = t + m * TT;
                    v[m] = {T(0), T(0)};
                    if (p < n) {
                        const cplx<T> w = tw_load(A, p);
                        const T a = at(p);
                        v[m] = {a * w.x, a * w.y};
                    }
                }
            }
            break;
    }
    if (rp.conj) {
#pragma unroll
        for (int m = 0; m < E; m++) v[m].y = -v[m].y;
    }
}

// REG_R2R post-processing (r2r_ir.rs:1390-1500): the FFT outputs at the thread's
// positions (v[m] at p = t + m TT) -> 0, 1 or 2 reals of the output line each.  With
// z = B[p] = W_8n^(4p+1), IV with n even writes k0 = 2p from r0 = Y z* and k1 = n-1-2p
// from conj(Y) W_8n^-(2 k1 + 1) = i conj(r0).
template <typename T, int N, int E, bool UNIT>
__device__ __forceinline__ void r2r_store_all(const RegParams &rp, T *out, int t, cplx<T> (&v)[E]) {
    constexpr int TT = N / E;
    const int64_t es = UNIT ? 1 : rp.dst.es;
    const int n = rp.r2r_n;
    const bool dst = rp.r2r_kind >= 4;
    const T s = T(rp.scale);
    const cplx<T> *A = reinterpret_cast<const cplx<T> *>(rp.tw2);
    const cplx<T> *B = A + N;
    if (rp.conj) {
#pragma unroll
        for (int m = 0; m < E; m++) v[m].y = -v[m].y;
    }
    auto put = [&](int k, T x) { __stcs(out + (int64_t)k * es, x * s); };
    switch (rp.r2r_kind & 3) {
        case 0:
#pragma unroll
            for (int m = 0; m < E; m++) {
                const int p = t + m * TT;
                if (!dst) {
                    if (p < n) put(p, v[m].x);
                } else if (p >= 1 && p <= n) {
                    put(p - 1, -v[m].y);
                }
            }
            break;
        case 1:
#pragma unroll
            for (int m = 0; m < E; m++) {
                const int p = t + m * TT;
                const cplx<T> w = tw_load(A, p);
                put(dst ? n - 1 - p : p, T(2) * (v[m].x * w.x - v[m].y * w.y));
            }
            break;
        case 2:
#pragma unroll
            for (int m = 0; m < E; m++) {
                const int p = t + m * TT;
                const int k = 2 * p < n ? 2 * p : 2 * n - 2 * p - 1;
                put(k, (dst && (k & 1)) ? -v[m].x : v[m].x);
            }
            break;
        default:
            if ((n & 1) == 0) {
#pragma unroll
                for (int m = 0; m < E; m++) {
                    const int p = t + m * TT;
                    const cplx<T> z = tw_load(B, p);
                    const cplx<T> r0 = mul(v[m], cplx<T>{z.x, -z.y});
                    put(2 * p, T(2) * (dst ? r0.y : r0.x));
                    put(n - 1 - 2 * p, T(2) * (dst ? r0.x : r0.y));
                }
            } else {
#pragma unroll
                for (int m = 0; m < E; m++) {
                    const int p = t + m * TT;
                    if (p < n) {
                        const cplx<T> r = mul(v[m], tw_load(B, p));
                        put(p, T(2) * (dst ? -r.y : r.x));
                    }
                }
            }
            break;
    }
}

// REG_R2R_HALF (N = h, the line holds n = 2h reals).  The II/III reductions of
// r2r_ir.rs:1282-1500 run a real length-n sequence through a complex FFT; here that
// sequence goes through the even-half algebra of the real FFT (real_ir.rs:1002-1013,
// 1087-1100) so the FFT has length h.  With A = W_n^k and B = W_4n^k (k = 0..h):
//   II:  z[p] = (v[2p], v[2p+1]) of the even-odd reorder v (odd sources negated for DST);
//        after FFT_h, V[p] = 1/2((Z[p] + conj Z[h-p]) - i A[p] (Z[p] - conj Z[h-p])) and
//        u = B[p] V[p] give X[p] = 2 Re u, X[n-p] = -2 Im u (DST: X at n-1-k).
//   III: V[k] = (a_k - i b_k) conj B[k] (a, b = x[k], x[n-k]; DST x[n-1-k], x[k-1]);
//        Z[p] = (V[p] + conj V[h-p]) + i conj A[p] (V[p] - conj V[h-p]); the inverse FFT_h
//        gives v[2p] + i v[2p+1], stored unreordered (odd outputs negated for DST).
template <typename T, int N, int E, typename At>
__device__ __forceinline__ void r2r_half_load_all(const RegParams &rp, At at, int t, cplx<T> (&v)[E]) {
    constexpr int TT = N / E;
    constexpr int n = 2 * N;
    const bool dst = rp.r2r_kind >= 4;
    const cplx<T> *A = reinterpret_cast<const cplx<T> *>(rp.tw2);
    const cplx<T> *B = A + (N + 1);
    if ((rp.r2r_kind & 3) == 1) {
        auto src = [&](int mm) { return mm < N ? 2 * mm : 2 * (n - mm) - 1; };
#pragma unroll
        for (int m = 0; m < E; m++) {
            const int p = t + m * TT;
            const int s0 = src(2 * p), s1 = src(2 * p + 1);
            T a = at(s0), b = at(s1);
            if (dst) {
                if (s0 & 1) a = -a;
                if (s1 & 1) b = -b;
            }
            v[m] = {a, b};
        }
    } else {
        auto Vk = [&](int k) {
            const T a = dst ? at(n - 1 - k) : at(k);
            const T b = k == 0 ? T(0) : (dst ? at(k - 1) : at(n - k));
            const cplx<T> w = tw_load(B, k);
            return mul(cplx<T>{a, -b}, cplx<T>{w.x, -w.y});
        };
#pragma unroll
        for (int m = 0; m < E; m++) {
            const int p = t + m * TT;
            const cplx<T> vp = Vk(p), vq = Vk(N - p);
            const cplx<T> sm = {vp.x + vq.x, vp.y - vq.y}, df = {vp.x - vq.x, vp.y + vq.y};
            const cplx<T> wa = tw_load(A, p);
            const cplx<T> r = mul(cplx<T>{wa.x, -wa.y}, df);
            v[m] = {sm.x - r.y, sm.y + r.x};
        }
    }
    if (rp.conj) {
#pragma unroll
        for (int m = 0; m < E; m++) v[m].y = -v[m].y;
    }
}

template <typename T, int N, int E>
__device__ __forceinline__ void r2r_half_epilogue(const RegParams &rp, cplx<T> (&v)[E], int t, cplx<T> *sline,
                                                  T *out, bool valid) {
    constexpr int TT = N / E;
    constexpr int n = 2 * N;
    const bool dst = rp.r2r_kind >= 4;
    const T s = T(rp.scale);
    const cplx<T> *A = reinterpret_cast<const cplx<T> *>(rp.tw2);
    const cplx<T> *B = A + (N + 1);
    if ((rp.r2r_kind & 3) == 1) {
        __syncthreads();  // the last stage's shared-memory reads are done
#pragma unroll
        for (int m = 0; m < E; m++) sline[pad<N>(t + m * TT)] = v[m];
        __syncthreads();
        if (!valid) return;
        auto put = [&](int k, T x) { __stcs(out + (dst ? n - 1 - k : k), x * s); };
        auto post = [&](cplx<T> a, cplx<T> bc, int kk) {
            const cplx<T> b = {bc.x, -bc.y};
            const cplx<T> r = mul(tw_load(A, kk), cplx<T>{a.x - b.x, a.y - b.y});
            return cplx<T>{T(0.5) * (a.x + b.x + r.y), T(0.5) * (a.y + b.y - r.x)};
        };
#pragma unroll
        for (int m = 0; m < E; m++) {
            const int p = t + m * TT;
            const cplx<T> zq = sline[pad<N>((N - p) & (N - 1))];
            const cplx<T> u = mul(tw_load(B, p), post(v[m], zq, p));
            put(p, T(2) * u.x);
            if (p != 0) put(n - p, T(-2) * u.y);
            if (p == 0) put(N, T(2) * mul(tw_load(B, N), post(v[m], v[m], N)).x);
        }
    } else {
        if (!valid) return;
        auto put = [&](int mm, T x) {
            const int k = mm < N ? 2 * mm : 2 * n - 2 * mm - 1;
            __stcs(out + k, ((dst && (k & 1)) ? -x : x) * s);
        };
#pragma unroll
        for (int m = 0; m < E; m++) {
            const int p = t + m * TT;
            cplx<T> z = v[m];
            if (rp.conj) z.y = -z.y;
            put(2 * p, z.x);
            put(2 * p + 1, z.y);
        }
    }
}

// Store of one output point at line position p (last stage), per data mode.
template <typename T, int N, int MODE>
__device__ __forceinline__ void store_point(const RegParams &rp, const LineIO &io, int p, cplx<T> y) {
    if (MODE == REG_C2C) {
        const T s = T(rp.scale);
        st_c<T>(rp.out, io.out_base + (int64_t)p * rp.dst.es, cplx<T>{y.x * s, rp.conj ? -y.y * s : y.y * s});
    } else if (MODE == REG_C2C_PEER) {
        // owner rank r of logical position p; the point lands in r's exchange buffer
        const T s = T(rp.scale);
        const int r = (int)((__umulhi((uint32_t)p, rp.peer.div.m) + (uint32_t)p) >> rp.peer.div.s);
        st_c<T>(rp.peer.ptr[r], io.out_base + (int64_t)p * rp.dst.es + rp.peer.off - (int64_t)r * rp.peer.sub,
                cplx<T>{y.x * s, rp.conj ? -y.y * s : y.y * s});
    } else if (MODE == REG_C2R_HALF) {
        // (x[2p], x[2p+1]) as one complex pair, conjugated back from the inverse trick
        const T s = T(rp.scale);
        st_c<T>(rp.out, io.out_base + p, cplx<T>{y.x * s, -y.y * s});
    } else if (MODE == REG_BLU_A) {
        const int64_t pos = io.out_pos0 + (int64_t)p * rp.dst.es;
        st_c<T>(rp.out, io.out_base + (int64_t)p * rp.dst.es,
                mul(y, tw_load(reinterpret_cast<const cplx<T> *>(rp.tw3), pos)));
    } else if (MODE == REG_BLU_C) {
        const int64_t n = io.out_pos0 + (int64_t)p * rp.dst.es;
        if (n < rp.n) {
            const T s = T(rp.scale);
            const cplx<T> r = mul(cplx<T>{y.x, -y.y}, tw_load(reinterpret_cast<const cplx<T> *>(rp.tw2), n));
            st_c<T>(rp.out, io.out_base + (int64_t)p * rp.dst.es, cplx<T>{r.x * s, rp.conj ? -r.y * s : r.y * s});
        }
    } else if (MODE == REG_R2C_FULL) {
        if (p <= N / 2) st_c<T>(rp.out, io.out_base + (int64_t)p * rp.dst.es, y);
    } else {
        __stcs(reinterpret_cast<T *>(rp.out) + io.out_base + (int64_t)p * rp.dst.es, y.x * T(rp.scale));
    }
}

// One radix-R stage with span P (product of the radices before it).  Its twiddles
// W_{P R}^{j q} are read from the stage's transposed table (row q-1 holds the P values
// of j, so a warp's loads are contiguous) at offset OFF; only the power-of-two rows
// are read and w_q = w_{q - lowbit(q)} * w_{lowbit(q)} forms the rest (at most three
// products deep).
template <typename T, int N, int E, int MODE, int R, int P, int OFF, bool FIRST, bool LAST>
__device__ __forceinline__ void stage(cplx<T> (&v)[E], int t, cplx<T> *sline, const cplx<T> *tw, const RegParams &rp,
                                      const LineIO &io) {
    constexpr int TT = N / E;
    constexpr int NB = E / R;  // butterflies per thread
    if (!FIRST) {
        __syncthreads();  // previous stage's outputs are visible
#pragma unroll
        for (int k = 0; k < NB; k++)
#pragma unroll
            for (int q = 0; q < R; q++) v[k + q * NB] = sline[pad<N>(t + k * TT + q * (N / R))];
        if (!LAST) __syncthreads();  // every thread has read before anyone overwrites
    }
#pragma unroll
    for (int k = 0; k < NB; k++) {
        cplx<T> x[R];
#pragma unroll
        for (int q = 0; q < R; q++) x[q] = v[k + q * NB];
        const int b = t + k * TT;
        const int j = b % P;
        if (P > 1) {
            cplx<T> w[R];
#pragma unroll
            for (int q = 1; q < R; q++) {
                if ((q & (q - 1)) == 0) {
                    w[q] = tw_load(tw, OFF + (q - 1) * P + j);
                } else {
                    const int lb = q & (-q);
                    w[q] = mul(w[q - lb], w[lb]);
                }
            }
#pragma unroll
            for (int q = 1; q < R; q++) x[q] = mul(x[q], w[q]);
        }
        dft<R, T>(x);
        if (LAST && (MODE == REG_R2C_HALF || MODE == REG_CONV || MODE == REG_R2R || MODE == REG_R2R_HALF)) {
            // output q of butterfly k sits at position t + (k + q NB) TT: back into v for
            // the post-processing epilogue
#pragma unroll
            for (int q = 0; q < R; q++) v[k + q * NB] = x[q];
        } else if (LAST) {
            if (io.valid) {
#pragma unroll
                for (int q = 0; q < R; q++) store_point<T, N, MODE>(rp, io, b + q * (N / R), x[q]);
            }
        } else {
            const int e0 = (b - j) * R + j;
#pragma unroll
            for (int q = 0; q < R; q++) sline[pad<N>(e0 + q * P)] = x[q];
        }
    }
}

template <typename T, int N, int E, int MODE, int P, int OFF, bool FIRST, int R, int... Rest>
__device__ __forceinline__ void stages(cplx<T> (&v)[E], int t, cplx<T> *sline, const cplx<T> *tw, const RegParams &rp,
                                       const LineIO &io) {
    constexpr bool LAST = sizeof...(Rest) == 0;
    stage<T, N, E, MODE, R, P, OFF, FIRST, LAST>(v, t, sline, tw, rp, io);
    // the first stage (P = 1) has no twiddles and no table rows
    constexpr int NEXT_OFF = OFF + (P > 1 ? (R - 1) * P : 0);
    if constexpr (!LAST) stages<T, N, E, MODE, P * R, NEXT_OFF, false, Rest...>(v, t, sline, tw, rp, io);
}

// REG_C2R_HALF pre-processing of position p from the h+1 bins X (accessor at(j)):
// Z[p] = s (X[p] + conj X[h-p] + i conj(W_2h^p) (X[p] - conj X[h-p])), conjugated for
// the inverse-by-forward trick.
template <typename T, int N, typename At>
__device__ __forceinline__ cplx<T> c2r_half_point(const RegParams &rp, At at, int p) {
    cplx<T> x = at(p);
    cplx<T> mc = at(N - p);
    if (p == 0 && rp.real_ends) x.y = mc.y = T(0);  // X[0], X[h]
    const cplx<T> wv = tw_load(reinterpret_cast<const cplx<T> *>(rp.tw2), p);
    const cplx<T> mm = {mc.x, -mc.y};
    const cplx<T> d = {x.x - mm.x, x.y - mm.y};
    const cplx<T> r = mul(cplx<T>{wv.x, -wv.y}, d);
    const T sc = T(rp.scale2);
    return {sc * (x.x + mm.x - r.y), -(sc * (x.y + mm.y + r.x))};
}

// REG_R2C_HALF post-processing: X[k] = 1/2 ((Z[k] + conj Z[h-k]) - i W_2h^k (Z[k] -
// conj Z[h-k])), k = 0..h.  Z[h-k] belongs to another thread, so Z goes through the
// line's shared-memory slot once.
template <typename T, int N, int E>
__device__ __forceinline__ void r2c_half_epilogue(const RegParams &rp, const cplx<T> (&v)[E], int t,
                                                  cplx<T> *sline, int64_t out_base, bool valid) {
    constexpr int TT = N / E;
    __syncthreads();  // the last stage's shared-memory reads are done
#pragma unroll
    for (int m = 0; m < E; m++) sline[pad<N>(t + m * TT)] = v[m];
    __syncthreads();
    if (!valid) return;
    const cplx<T> *w2 = reinterpret_cast<const cplx<T> *>(rp.tw2);
    auto post = [&](cplx<T> a, cplx<T> bc, int kk) {
        const cplx<T> b = {bc.x, -bc.y};
        const cplx<T> r = mul(tw_load(w2, kk), cplx<T>{a.x - b.x, a.y - b.y});
        return cplx<T>{T(0.5) * (a.x + b.x + r.y), T(0.5) * (a.y + b.y - r.x)};
    };
#pragma unroll
    for (int m = 0; m < E; m++) {
        const int p = t + m * TT;
        const cplx<T> zk2 = sline[pad<N>((N - p) & (N - 1))];
        st_c<T>(rp.out, out_base + p, post(v[m], zk2, p));
        if (p == 0) st_c<T>(rp.out, out_base + N, post(v[m], v[m], N));
    }
}

template <typename T, int N, int E, int G, int MODE, bool STRIDED, int... Rs>
__global__ void __launch_bounds__(G *(N / E)) reg_fft_kernel(const __grid_constant__ RegParams rp) {
    constexpr int TT = N / E;
    constexpr int LS = reg_ls<T>(N, E, G, STRIDED);  // line stride in shared memory
    extern __shared__ __align__(16) unsigned char smem_raw[];
    int g, t;
    if (STRIDED) {
        g = threadIdx.x % G;
        t = threadIdx.x / G;
    } else {
        g = threadIdx.x / TT;
        t = threadIdx.x - g * TT;
    }
    const int64_t line = (int64_t)blockIdx.x * G + g;
    LineIO io;
    io.valid = line < rp.nlines;
    {
        const int64_t o = rp.ni == 1 ? line : line / rp.ni;
        const int64_t i = line - o * rp.ni;
        io.in_base = o * rp.src.os + i * rp.src.is;
        io.out_base = o * rp.dst.os + i * rp.dst.is;
        io.in_pos0 = i * rp.src.is;
        io.out_pos0 = i * rp.dst.is;
    }
    cplx<T> *sline = reinterpret_cast<cplx<T> *>(smem_raw) + g * LS;
    const cplx<T> *tw = reinterpret_cast<const cplx<T> *>(rp.tw);
    cplx<T> v[E];
    if (MODE == REG_R2R && io.valid) {
        const T *x = reinterpret_cast<const T *>(rp.in) + io.in_base;
        const int64_t es = STRIDED ? rp.src.es : 1;
        r2r_load_all<T, N, E>(rp, [&](int j) { return __ldcs(x + (int64_t)j * es); }, t, v);
    } else if (MODE == REG_R2R_HALF && io.valid) {
        const T *x = reinterpret_cast<const T *>(rp.in) + io.in_base;
        r2r_half_load_all<T, N, E>(rp, [&](int j) { return __ldcs(x + j); }, t, v);
    } else if (MODE != REG_R2R && MODE != REG_R2R_HALF && io.valid) {
#pragma unroll
        for (int m = 0; m < E; m++) {
            const int p = t + m * TT;
            if (MODE == REG_CONV) {
                v[m] = ld_c<T>(rp.in, io.in_base + (int64_t)p * rp.src.es);
            } else if (MODE == REG_BLU_A) {
                const int64_t n = io.in_pos0 + (int64_t)p * rp.src.es;
                v[m] = {T(0), T(0)};
                if (n < rp.n) {
                    const cplx<T> w = ld_c<T>(rp.in, io.in_base + (int64_t)p * rp.src.es);
                    v[m] = mul(cplx<T>{w.x, rp.conj ? -w.y : w.y},
                               tw_load(reinterpret_cast<const cplx<T> *>(rp.tw2), n));
                }
            } else if (MODE == REG_BLU_C) {
                const cplx<T> w = ld_c<T>(rp.in, io.in_base + (int64_t)p * rp.src.es);
                v[m] = {w.x, -w.y};
            } else if (MODE == REG_C2C || MODE == REG_C2C_PEER || MODE == REG_R2C_HALF) {
                const cplx<T> w = ld_c<T>(rp.in, io.in_base + (int64_t)p * rp.src.es);
                v[m] = {w.x, rp.conj ? -w.y : w.y};
            } else if (MODE == REG_C2R_HALF) {
                v[m] = c2r_half_point<T, N>(rp, [&](int j) { return ld_c<T>(rp.in, io.in_base + j); }, p);
            } else if (MODE == REG_R2C_FULL) {
                v[m] = {__ldcs(reinterpret_cast<const T *>(rp.in) + io.in_base + (int64_t)p * rp.src.es), T(0)};
            } else {
                // Hermitian mirror X[p] = conj(X[N - p]) for p > N/2; the inverse transform
                // runs on conj(X), so the stored half is conjugated and the mirror is not
                const int q = p <= N / 2 ? p : N - p;
                const cplx<T> w = ld_c<T>(rp.in, io.in_base + (int64_t)q * rp.src.es);
                v[m] = {w.x, p <= N / 2 ? -w.y : w.y};
            }
        }
    } else {
#pragma unroll
        for (int m = 0; m < E; m++) v[m] = {T(0), T(0)};
    }
    if constexpr (MODE == REG_CONV) {
        // forward FFT (outputs back in v at positions t + m TT), spectrum multiply with the
        // convolution policy, then the inverse FFT as conj(FFT(conj .)) whose store
        // conjugates and scales (rp.conj = 1, rp.scale = 1/N)
        stages<T, N, E, REG_CONV, 1, 0, true, Rs...>(v, t, sline, tw, rp, io);
        const cplx<T> *spec = reinterpret_cast<const cplx<T> *>(rp.tw2);
        const int64_t o = rp.ni == 1 ? line : line / rp.ni;
        const int64_t i = line - o * rp.ni;
        const int64_t base = i + o * rp.conv_om;
#pragma unroll
        for (int m = 0; m < E; m++) {
            const int p = t + m * TT;
            cplx<T> x = v[m];
            if (rp.conv_flags & F_CONJ_IN) x.y = -x.y;
            if (io.valid) x = mul(x, tw_load(spec, base + (int64_t)p * rp.conv_em));
            if (rp.conv_flags & F_NORMALIZE) {
                const T r = T(1) / sqrt(x.x * x.x + x.y * x.y);
                x.x *= r;
                x.y *= r;
            }
            if (rp.conv_flags & F_CONJ_OUT) x.y = -x.y;
            v[m] = x;
        }
        __syncthreads();  // the forward FFT's last shared-memory reads are done
        stages<T, N, E, REG_C2C, 1, 0, true, Rs...>(v, t, sline, tw, rp, io);
        return;
    }
    stages<T, N, E, MODE, 1, 0, true, Rs...>(v, t, sline, tw, rp, io);
    if (MODE == REG_R2R && io.valid) r2r_store_all<T, N, E, !STRIDED>(rp, reinterpret_cast<T *>(rp.out) + io.out_base, t, v);
    // peer stores are visible system-wide before the rank's exchange signal
    if (MODE == REG_C2C_PEER) __threadfence_system();
    if (MODE == REG_R2C_HALF) r2c_half_epilogue<T, N, E>(rp, v, t, sline, io.out_base, io.valid);
    if (MODE == REG_R2R_HALF)
        r2r_half_epilogue<T, N, E>(rp, v, t, sline, reinterpret_cast<T *>(rp.out) + io.out_base, io.valid);
}

// ---- persistent variant: bulk-copy prefetch of the next line group -------------------
// Dense contiguous lines (REG_C2C: N complex points; REG_C2R_HALF: N+1 bins; REG_R2R:
// the real line of rp.r2r_n values), every group's bytes a multiple of 16:
// each CTA loops over groups of G lines.  One thread fetches the group with cp.async.bulk into a shared
// buffer, tracked by an mbarrier; as soon as every thread has taken its points from the
// buffer it fetches the CTA's next group, so the next load overlaps the radix stages and
// the stores of the current one.  Waits are bounded: on expiry the kernel records error
// bit 64 and stops.

__device__ __forceinline__ unsigned smem_addr(const void *p) { return (unsigned)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void bulk_fetch(void *dst, const void *src, unsigned bytes, uint64_t *bar) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ bool bar_wait(uint64_t *bar, unsigned parity) {
    for (int i = 0; i < (1 << 22); i++) {
        unsigned done;
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
            : "=r"(done)
            : "r"(smem_addr(bar)), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

template <typename T, int N, int E, int G, int MINB, int MODE, int... Rs>
__global__ void __launch_bounds__(G *(N / E), MINB) reg_fft_persistent(const __grid_constant__ RegParams rp) {
    constexpr int TT = N / E;
    constexpr int LS = reg_ls<T>(N, E, G, false);
    // bytes of one line in the input: N complex (C2C, R2C_HALF), N+1 bins (C2R_HALF), or
    // r2r_n reals (R2R, at most 2N of them)
    const unsigned LINE_BYTES = (MODE == REG_R2R || MODE == REG_R2R_HALF) ? (unsigned)(rp.r2r_n * sizeof(T))
                                : MODE == REG_C2R_HALF ? (unsigned)((N + 1) * sizeof(cplx<T>))
                                                       : (unsigned)(N * sizeof(cplx<T>));
    const unsigned GROUP_BYTES = G * LINE_BYTES;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem_raw);
    cplx<T> *buf = reinterpret_cast<cplx<T> *>(smem_raw + 128);
    cplx<T> *xch = buf + G * (N + 1);
    const int g = threadIdx.x / TT, t = threadIdx.x - g * TT;
    cplx<T> *sline = xch + g * LS;
    const cplx<T> *tw = reinterpret_cast<const cplx<T> *>(rp.tw);
    const int64_t ngroups = (rp.nlines + G - 1) / G;
    auto group_bytes = [&](int64_t grp) {
        const int64_t lines = rp.nlines - grp * G;
        return lines >= G ? GROUP_BYTES : (unsigned)(lines * LINE_BYTES);
    };
    auto group_src = [&](int64_t grp) {
        return reinterpret_cast<const unsigned char *>(rp.in) + grp * (int64_t)GROUP_BYTES;
    };
    if (threadIdx.x == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(bar)) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    int64_t grp = blockIdx.x;
    bool in_flight = false;
    if (threadIdx.x == 0 && grp < ngroups) {
        bulk_fetch(buf, group_src(grp), group_bytes(grp), bar);
        in_flight = true;
    }
    unsigned parity = 0;
    for (; grp < ngroups; grp += gridDim.x) {
        if (!bar_wait(bar, parity)) {
            if (threadIdx.x == 0) atomicOr(rp.err, 64);
            break;
        }
        parity ^= 1u;
        in_flight = false;
        const int64_t line = grp * G + g;
        LineIO io;
        io.valid = line < rp.nlines;
        io.in_base = line * rp.src.os;
        io.out_base = line * rp.dst.os;
        cplx<T> v[E];
        if (MODE == REG_R2R) {
            const T *xs = reinterpret_cast<const T *>(buf) + g * rp.r2r_n;
            r2r_load_all<T, N, E>(rp, [&](int j) { return xs[j]; }, t, v);
        } else if (MODE == REG_R2R_HALF) {
            const T *xs = reinterpret_cast<const T *>(buf) + g * rp.r2r_n;
            r2r_half_load_all<T, N, E>(rp, [&](int j) { return xs[j]; }, t, v);
        } else if (MODE == REG_C2R_HALF) {
            const cplx<T> *xs = buf + g * (N + 1);
#pragma unroll
            for (int m = 0; m < E; m++) v[m] = c2r_half_point<T, N>(rp, [&](int j) { return xs[j]; }, t + m * TT);
        } else {
#pragma unroll
            for (int m = 0; m < E; m++) {
                const cplx<T> w = buf[g * N + t + m * TT];
                v[m] = {w.x, rp.conj ? -w.y : w.y};
            }
        }
        __syncthreads();  // the group buffer is consumed
        const int64_t nxt = grp + gridDim.x;
        if (threadIdx.x == 0 && nxt < ngroups) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            bulk_fetch(buf, group_src(nxt), group_bytes(nxt), bar);
            in_flight = true;
        }
        stages<T, N, E, MODE, 1, 0, true, Rs...>(v, t, sline, tw, rp, io);
        if (MODE == REG_R2R && io.valid) r2r_store_all<T, N, E, true>(rp, reinterpret_cast<T *>(rp.out) + io.out_base, t, v);
        if (MODE == REG_R2C_HALF) r2c_half_epilogue<T, N, E>(rp, v, t, sline, io.out_base, io.valid);
        if (MODE == REG_R2R_HALF)
            r2r_half_epilogue<T, N, E>(rp, v, t, sline, reinterpret_cast<T *>(rp.out) + io.out_base, io.valid);
    }
    // never leave with a bulk copy still writing this CTA's shared memory
    if (threadIdx.x == 0 && in_flight && !bar_wait(bar, parity)) atomicOr(rp.err, 64);
}

// ---- Rader lines in registers ---------------------------------------------------------
// One thread per line of prime length P (the strided higher axes of the ND configs, e.g.
// the 17-point axis of [1024, 17, 65537]): the P points are loaded straight into
// registers (a warp reads 32 neighbouring lines of the same position: coalesced), and
// Rader's algorithm (rader_ir.rs: generator permutation, cyclic convolution of length
// P - 1 through the codelet FFT, x0 added back) runs without shared memory:
//   a[q] = x[g^q],  A = FFT(a),  X[0] = x[0] + A[0],
//   c = IFFT(A * FFT(b)),  b[q] = W_P^(g^-q),  X[g^-m] = x[0] + c[m],
// with the inverse FFT as conj(FFT(conj .)) and rp.tw = FFT(b) / (P - 1) (lower.cpp
// table_rader_line).  g is the smallest primitive root of P; the permutations are
// compile-time constants, so every register index folds.
__host__ __device__ constexpr int pow_mod(int g, int e, int p) {
    int r = 1;
    for (int k = 0; k < e; k++) r = r * g % p;
    return r;
}
__host__ __device__ constexpr int smallest_primitive_root(int p) {
    for (int g = 2; g < p; g++) {
        bool ok = true;
        for (int e = 1; e < p - 1; e++)
            if (pow_mod(g, e, p) == 1) ok = false;
        if (ok) return g;
    }
    return 1;
}

template <typename T, int P, int G>
__global__ void __launch_bounds__(G) reg_rader_kernel(const __grid_constant__ RegParams rp) {
    constexpr int L = P - 1;
    constexpr int g = smallest_primitive_root(P);
    constexpr int ginv = pow_mod(g, P - 2, P);  // g^-1 mod P
    const int64_t line = (int64_t)blockIdx.x * G + threadIdx.x;
    if (line >= rp.nlines) return;
    const int64_t o = rp.ni == 1 ? line : line / rp.ni;
    const int64_t i = line - o * rp.ni;
    const int64_t ib = o * rp.src.os + i * rp.src.is, ob = o * rp.dst.os + i * rp.dst.is;
    cplx<T> x[P];
#pragma unroll
    for (int p = 0; p < P; p++) {
        x[p] = ld_c<T>(rp.in, ib + (int64_t)p * rp.src.es);
        if (rp.conj) x[p].y = -x[p].y;
    }
    cplx<T> a[L];
#pragma unroll
    for (int q = 0; q < L; q++) a[q] = x[pow_mod(g, q, P)];
    dft<L, T>(a);
    const cplx<T> x0 = x[0];
    const cplx<T> X0 = {x0.x + a[0].x, x0.y + a[0].y};
    const cplx<T> *B = reinterpret_cast<const cplx<T> *>(rp.tw);
#pragma unroll
    for (int k = 0; k < L; k++) {
        const cplx<T> y = mul(a[k], tw_load(B, k));
        a[k] = {y.x, -y.y};
    }
    dft<L, T>(a);  // conj(c[m]) in a[m]
    const T s = T(rp.scale);
    auto put = [&](int k, cplx<T> v) {
        st_c<T>(rp.out, ob + (int64_t)k * rp.dst.es, cplx<T>{v.x * s, rp.conj ? -v.y * s : v.y * s});
    };
    put(0, X0);
#pragma unroll
    for (int m = 0; m < L; m++) put(pow_mod(ginv, m, P), cplx<T>{x0.x + a[m].x, x0.y - a[m].y});
}

}  // namespace regk

// ---- variant table ----------------------------------------------------------------

struct RegVariant {
    int is_double, n, mode, strided, threads, g;
    size_t smem;
    const void *fn;
    int radices[8];
    int persistent;  // reg_fft_persistent (grid sized to the resident CTAs)
};

#define RV(T, MODE, STR, N, E, G, ...)                                                                      \
    {sizeof(T) == 8, N, MODE, STR, G *(N / E), G, (size_t)G * regk::reg_ls<T>(N, E, G, STR) * sizeof(T) * 2,  \
     (const void *)regk::reg_fft_kernel<T, N, E, G, MODE, STR, __VA_ARGS__>, {__VA_ARGS__}, 0}
// persistent contiguous lines: barrier slot + one group buffer + the exchange buffer
#define RVP(T, MODE, N, E, G, MINB, ...)                                                                    \
    {sizeof(T) == 8, N, MODE, 0, G *(N / E), G,                                                             \
     128 + (size_t)G * (N + 1) * sizeof(T) * 2 + (size_t)G * regk::reg_ls<T>(N, E, G, false) * sizeof(T) * 2, \
     (const void *)regk::reg_fft_persistent<T, N, E, G, MINB, MODE, __VA_ARGS__>, {__VA_ARGS__}, 1}
#define RVP_ALL(T, MODE)                                                                                    \
    RVP(T, MODE, 256, 16, 16, 3, 16, 16), RVP(T, MODE, 512, 16, 8, 3, 16, 16, 2),                           \
        RVP(T, MODE, 1024, 16, 4, 3, 16, 16, 4), RVP(T, MODE, 2048, 16, 2, 3, 16, 16, 8),                   \
        RVP(T, MODE, 4096, 16, 1, 3, 16, 16, 16)

// contiguous lines, all modes
#define RV_CONTIG(T, MODE)                                                                                  \
    RV(T, MODE, false, 16, 16, 64, 16), RV(T, MODE, false, 32, 16, 64, 16, 2),                            \
        RV(T, MODE, false, 64, 16, 32, 16, 4), RV(T, MODE, false, 128, 16, 16, 16, 8),                   \
        RV(T, MODE, false, 256, 16, 16, 16, 16), RV(T, MODE, false, 512, 16, 8, 16, 16, 2),              \
        RV(T, MODE, false, 1024, 16, 4, 16, 16, 4), RV(T, MODE, false, 2048, 16, 2, 16, 16, 8),          \
        RV(T, MODE, false, 4096, 16, 1, 16, 16, 16), RV(T, MODE, false, 8192, 16, 1, 16, 16, 16, 2)

// strided (higher-axis) lines, the slab exchange twins of the strided C2C variants
#define RV_STRIDED(T, MODE)                                                                                 \
    RV(T, MODE, true, 16, 16, 32, 16), RV(T, MODE, true, 32, 16, 32, 16, 2),                               \
        RV(T, MODE, true, 64, 16, (sizeof(T) == 8 ? 16 : 32), 16, 4),                                        \
        RV(T, MODE, true, 128, 16, (sizeof(T) == 8 ? 16 : 32), 16, 8), RV(T, MODE, true, 256, 16, 16, 16, 16), \
        RV(T, MODE, true, 512, 16, (sizeof(T) == 8 ? 8 : 16), 16, 16, 2),                                    \
        RV(T, MODE, true, 1024, 16, (sizeof(T) == 8 ? 4 : 16), 16, 16, 4),                                   \
        RV(T, MODE, true, 2048, 16, (sizeof(T) == 8 ? 4 : 8), 16, 16, 8),                                    \
        RV(T, MODE, true, 4096, 16, (sizeof(T) == 8 ? 2 : 4), 16, 16, 16)

static const RegVariant kRegVariants[] = {
    RV_CONTIG(float, REG_C2C),
    RV_CONTIG(double, REG_C2C),
    RV_CONTIG(float, REG_R2C_FULL),
    RV_CONTIG(double, REG_R2C_FULL),
    RV_CONTIG(float, REG_C2R_FULL),
    RV_CONTIG(double, REG_C2R_FULL),
    RV_CONTIG(float, REG_C2C_PEER),
    RV_CONTIG(double, REG_C2C_PEER),
    RV_CONTIG(float, REG_R2C_HALF),
    RV_CONTIG(double, REG_R2C_HALF),
    RV_CONTIG(float, REG_C2R_HALF),
    RV_CONTIG(double, REG_C2R_HALF),
    // strided (higher-axis) C2C lines: G neighbouring lines per CTA
    RV(float, REG_C2C, true, 16, 16, 32, 16), RV(float, REG_C2C, true, 32, 16, 32, 16, 2),
    RV(float, REG_C2C, true, 64, 16, 32, 16, 4), RV(float, REG_C2C, true, 128, 16, 32, 16, 8),
    RV(float, REG_C2C, true, 256, 16, 16, 16, 16), RV(float, REG_C2C, true, 512, 32, 16, 32, 16),
    RV(float, REG_C2C, true, 1024, 32, 16, 32, 32), RV(float, REG_C2C, true, 2048, 16, 8, 16, 16, 8),
    RV(float, REG_C2C, true, 4096, 16, 4, 16, 16, 16),
    RV(double, REG_C2C, true, 16, 16, 32, 16), RV(double, REG_C2C, true, 32, 16, 32, 16, 2),
    RV(double, REG_C2C, true, 64, 16, 16, 16, 4), RV(double, REG_C2C, true, 128, 16, 16, 16, 8),
    RV(double, REG_C2C, true, 256, 16, 16, 16, 16), RV(double, REG_C2C, true, 512, 16, 8, 16, 16, 2),
    RV(double, REG_C2C, true, 1024, 16, 4, 16, 16, 4), RV(double, REG_C2C, true, 2048, 16, 4, 16, 16, 8),
    RV(double, REG_C2C, true, 4096, 16, 2, 16, 16, 16),
    // Rader lines in registers (one thread per line, strided higher axes)
    {0, 17, REG_RADER_LINE, 1, 128, 128, 0, (const void *)regk::reg_rader_kernel<float, 17, 128>, {16}, 0},
    {1, 17, REG_RADER_LINE, 1, 128, 128, 0, (const void *)regk::reg_rader_kernel<double, 17, 128>, {16}, 0},
    // four-step Bluestein column passes of M = 324 x 405 (the 65537-point axes of BASELINE config 4)
    RV(float, REG_BLU_A, true, 324, 18, 16, 2, 2, 9, 9), RV(float, REG_BLU_C, true, 324, 18, 16, 2, 2, 9, 9),
    // (f64 columns measured slower in the register kernel than on the generic passes:
    // 65537 x 2048 f64 23.6 vs 23.0 ms per step, so f64 keeps the generic passes)
    RV_STRIDED(float, REG_C2C_PEER),
    RV_STRIDED(double, REG_C2C_PEER),
    RV_STRIDED(float, REG_CONV),
    RV_STRIDED(double, REG_CONV),
    // DCT / DST reductions fused into the FFT of the axis
    RV_CONTIG(float, REG_R2R),
    RV_CONTIG(double, REG_R2R),
    RV_STRIDED(float, REG_R2R),
    RV_STRIDED(double, REG_R2R),
    RV_CONTIG(float, REG_R2R_HALF),
    // persistent twins of the contiguous C2C variants (bulk-copy prefetch)
    // (blocks per SM asked of the register allocator: the shared-memory limit)
    RVP_ALL(float, REG_C2C),
    RVP_ALL(float, REG_R2R),
    RVP_ALL(float, REG_C2R_HALF),
    RVP_ALL(float, REG_R2R_HALF),
    // (f64 groups need twice the buffer and registers: one CTA per SM, slower than the
    // ordinary kernel's two, so f64 keeps the ordinary variants)
};
#undef RV_CONTIG
#undef RV_STRIDED
#undef RVP_ALL
#undef RVP
#undef RV

int reg_variant_for(bool is_double, size_t n, int mode, bool strided) {
    for (int i = 0; i < (int)(sizeof(kRegVariants) / sizeof(kRegVariants[0])); i++) {
        const RegVariant &v = kRegVariants[i];
        if (v.is_double == (int)is_double && (size_t)v.n == n && v.mode == mode && v.strided == (int)strided &&
            !v.persistent)
            return i;
    }
    return -1;
}

// The persistent twin of a contiguous C2C or R2R variant (same mode, precision, length,
// radices and lines per CTA), or -1.
int reg_variant_persistent_twin(int v) {
    const RegVariant &a = kRegVariants[v];
    if ((a.mode != REG_C2C && a.mode != REG_R2R && a.mode != REG_R2R_HALF && a.mode != REG_C2R_HALF) || a.strided ||
        a.persistent)
        return -1;
    for (int i = 0; i < (int)(sizeof(kRegVariants) / sizeof(kRegVariants[0])); i++) {
        const RegVariant &b = kRegVariants[i];
        if (b.persistent && b.mode == a.mode && b.is_double == a.is_double && b.n == a.n && b.g == a.g &&
            b.smem <= 232448)
            return i;
    }
    return -1;
}

// Radix sequence of a variant (0-terminated in the table); returns the stage count.
int reg_variant_radices(int v, int *out) {
    int n = 0;
    while (n < 8 && kRegVariants[v].radices[n]) {
        out[n] = kRegVariants[v].radices[n];
        n++;
    }
    return n;
}

int reg_variant_lines_per_cta(int v) { return kRegVariants[v].g; }

int reg_variant_length(int v) { return kRegVariants[v].n; }

// The REG_C2C_PEER twin of a REG_C2C variant (same precision, length and layout), or -1.
int reg_variant_peer_twin(int v) {
    const RegVariant &a = kRegVariants[v];
    if (a.mode != REG_C2C) return -1;
    return reg_variant_for(a.is_double != 0, (size_t)a.n, REG_C2C_PEER, a.strided != 0);
}

void set_reg_kernel_smem_limits() {
    static unsigned long long done_mask = 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return;
    if (done_mask & (1ull << dev)) return;
    for (const RegVariant &v : kRegVariants)
        cudaFuncSetAttribute(v.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)v.smem);
    done_mask |= 1ull << dev;
}

// Resident CTAs of a persistent variant on the current device (cached per device).
static int64_t persistent_grid(int variant) {
    static int cache[64][sizeof(kRegVariants) / sizeof(kRegVariants[0])] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    int &c = cache[dev][variant];
    if (!c) {
        const RegVariant &v = kRegVariants[variant];
        int sms = 0, per = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, v.fn, v.threads, v.smem);
        c = std::max(1, sms) * std::max(1, per);
    }
    return c;
}

cudaError_t launch_reg(int variant, const RegParams &rp, cudaStream_t stream) {
    const RegVariant &v = kRegVariants[variant];
    int64_t grid = (rp.nlines + v.g - 1) / v.g;
    if (v.persistent) grid = std::min<int64_t>(grid, persistent_grid(variant));
    void *args[] = {const_cast<RegParams *>(&rp)};
    return cudaLaunchKernel(v.fn, dim3((unsigned)grid), dim3(v.threads), args, v.smem, stream);
}

}  // namespace b200fft
