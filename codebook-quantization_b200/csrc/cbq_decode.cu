// cbq_decode.cu -- the per-token transformer-block kernels around the
// compressed linear layers of a decode step (sm_100a): RMSNorm (with the
// residual add folded in), per-head q/k RMSNorm + rotary embedding + KV-cache
// write, and grouped-query attention of one new token against the cache.
//
// The math is HF transformers' Qwen3 (models/qwen3: Qwen3RMSNorm,
// apply_rotary_pos_emb with rotate_half, grouped-query attention with
// softmax scale d^-1/2).  Element-wise steps round to the activation dtype at
// the same points as the unfused torch sequence; reductions (sum of squares,
// softmax, the attention-weighted sum) accumulate in fp32.
#include <algorithm>
#include <climits>

#include "cbq_common.cuh"

namespace {

using namespace cbq;

template <typename T> __device__ __forceinline__ float ld(const T *p, int64_t i) { return to_f32(p[i]); }
template <typename T> __device__ __forceinline__ float rnd(float v) { return to_f32(from_f32<T>(v)); }

template <int NT>
__device__ __forceinline__ float block_sum(float v, float *red) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) red[w] = v;
    __syncthreads();
    float t = 0.f;
    if (w == 0) {
        t = l < NT / 32 ? red[l] : 0.f;
        t = warp_sum(t);
        if (l == 0) red[0] = t;
    }
    __syncthreads();
    t = red[0];
    __syncthreads();
    return t;
}

// ------------------------------------------------------------------ RMSNorm
// x[r] (+)= add[r] (rounded), out[r] = round(w * round(x * rsqrt(mean(x^2) + eps))).
template <typename T, int NT>
__global__ void __launch_bounds__(NT) k_rmsnorm(T *x, const T *add, int64_t n, const float *w, float eps,
                                                T *out) {
    __shared__ float red[32];
    pdl_launch_dependents();
    pdl_wait();
    const int64_t r = blockIdx.x;
    T *xr = x + r * n;
    const T *ar = add ? add + r * n : nullptr;
    T *orow = out + r * n;
    float ss = 0.f;
    for (int64_t i = threadIdx.x; i < n; i += NT) {
        float v = ld(xr, i);
        if (ar) {
            v = rnd<T>(v + ld(ar, i));
            xr[i] = from_f32<T>(v);
        }
        ss += v * v;
    }
    const float tot = block_sum<NT>(ss, red);
    const float scale = rsqrtf(tot / (float)n + eps);
    for (int64_t i = threadIdx.x; i < n; i += NT) {
        float v = rnd<T>(ld(xr, i) * scale);
        if (w) v = w[i] * v;
        orow[i] = from_f32<T>(v);
    }
}

// -------------------------------------- all-reduce + residual + RMSNorm
// The consumer of the peer-partial GEMV epilogue: wait until every rank s has
// delivered its partial rows to slot s (counts[s] >= epoch * expect; bounded,
// %globaltimer), then x[r] = round(x[r] + round(sum_s slot[s][r])) in rank
// order (every rank computes the same values) and out[r] = RMSNorm(x[r]).
template <typename T, int NT>
__global__ void __launch_bounds__(NT) k_rmsnorm_allreduce(T *x, const T *slots, const uint32_t *counts,
                                                          const uint32_t *epoch, uint32_t expect, int world,
                                                          int64_t rows, int64_t n, const float *w, float eps,
                                                          T *out, uint32_t *status) {
    __shared__ float red[32];
    __shared__ int late;
    pdl_launch_dependents();
    pdl_wait();
    // a wait that already gave up in this run: do not wait again
    if (threadIdx.x == 0) late = (status && (*(volatile uint32_t *)(status + CBQ_STATUS_FLAGS) & CBQ_FLAG_TIMEOUT)) ? 1 : 0;
    __syncthreads();
    if (late) return;
    if (threadIdx.x < world) {
        const uint32_t want = *epoch * expect;
        const uint64_t t0 = global_timer_ns();
        while (true) {
            uint32_t c;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(c) : "l"(counts + threadIdx.x) : "memory");
            if ((int32_t)(c - want) >= 0) break;
            if (global_timer_ns() - t0 > kWaitNs) {
                late = 1;
                break;
            }
            __nanosleep(64);
        }
    }
    __syncthreads();
    if (late) {
        if (threadIdx.x == 0 && blockIdx.x == 0) report(status, CBQ_FLAG_TIMEOUT, 0u);
        return;
    }
    __threadfence_system();
    const int64_t r = blockIdx.x;
    T *xr = x + r * n;
    T *orow = out + r * n;
    float ss = 0.f;
    for (int64_t i = threadIdx.x; i < n; i += NT) {
        float sum = 0.f;
        for (int p = 0; p < world; ++p) sum += ld(slots, ((int64_t)p * rows + r) * n + i);
        const float v = rnd<T>(ld(xr, i) + rnd<T>(sum));
        xr[i] = from_f32<T>(v);
        ss += v * v;
    }
    const float tot = block_sum<NT>(ss, red);
    const float scale = rsqrtf(tot / (float)n + eps);
    for (int64_t i = threadIdx.x; i < n; i += NT) {
        float v = rnd<T>(ld(xr, i) * scale);
        if (w) v = w[i] * v;
        orow[i] = from_f32<T>(v);
    }
}

// ------------------------------------------- q/k norm + rope + cache write
// One head held by a warp (lane l: elements [l*E, l*E + E), E = d/32):
// per-head RMSNorm with weight w (may be null), then rotate_half RoPE with the
// lane's cos / sin values c, sn of the position; rotate_half's partner of
// element i is i +- d/2, held by lane l ^ 16.  Rounds to T where the unfused
// torch sequence does.
template <typename T, int E>
__device__ __forceinline__ void qk_head(const float (&x0)[E], float eps, const float *w, const float (&c)[E],
                                        const float (&sn)[E], int lane, float (&o)[E]) {
    constexpr int D = 32 * E;
    float x[E];
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) ss += x0[e] * x0[e];
    ss = warp_sum(ss);
    const float scale = rsqrtf(ss / (float)D + eps);
#pragma unroll
    for (int e = 0; e < E; ++e) {
        x[e] = rnd<T>(x0[e] * scale);
        if (w) x[e] = rnd<T>(w[lane * E + e] * x[e]);
    }
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int i = lane * E + e;
        const float partner = __shfl_xor_sync(0xffffffffu, x[e], 16);
        const float rot = i < D / 2 ? -partner : partner;
        o[e] = rnd<T>(rnd<T>(x[e] * c[e]) + rnd<T>(rot * sn[e]));
    }
}

// The lane's cos / sin values of one table row, rounded to T as the torch
// sequence rounds them.
template <typename T, int E>
__device__ __forceinline__ void rope_row(const float *cr, const float *sr, int lane, float (&c)[E], float (&sn)[E]) {
#pragma unroll
    for (int e = 0; e < E; ++e) {
        c[e] = rnd<T>(cr[lane * E + e]);
        sn[e] = rnd<T>(sr[lane * E + e]);
    }
}

// One warp per head: heads [0, Hq) of q, then Hkv of k, then Hkv of v, for
// each of B rows.
template <typename T, int E>
__global__ void __launch_bounds__(256) k_qk_norm_rope(const T *q, const T *k, const T *v, int B, int Hq,
                                                      int Hkv, float eps, const float *qw, const float *kw,
                                                      const float *cosT, const float *sinT,
                                                      const int64_t *pos_dev, T *q_out, T *k_cache,
                                                      T *v_cache, int64_t L) {
    constexpr int D = 32 * E;
    pdl_launch_dependents();
    pdl_wait();
    const int gw = (int)((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    const int per_row = Hq + 2 * Hkv;
    if (gw >= B * per_row) return;
    const int b = gw / per_row, h = gw - b * per_row;
    const int64_t pos = *pos_dev;
    if (pos < 0 || pos >= L) return;                  // outside the cache: write nothing
    float x[E];
    const T *src;
    int kind, hh;
    if (h < Hq) { kind = 0; hh = h; src = q + ((int64_t)b * Hq + hh) * D; }
    else if (h < Hq + Hkv) { kind = 1; hh = h - Hq; src = k + ((int64_t)b * Hkv + hh) * D; }
    else { kind = 2; hh = h - Hq - Hkv; src = v + ((int64_t)b * Hkv + hh) * D; }
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = ld(src, lane * E + e);
    if (kind == 2) {
        T *dst = v_cache + (((int64_t)b * Hkv + hh) * L + pos) * D;
#pragma unroll
        for (int e = 0; e < E; ++e) dst[lane * E + e] = from_f32<T>(x[e]);
        return;
    }
    float o[E], c[E], sn[E];
    rope_row<T, E>(cosT + pos * D, sinT + pos * D, lane, c, sn);
    qk_head<T, E>(x, eps, kind == 0 ? qw : kw, c, sn, lane, o);
    T *dst = kind == 0 ? q_out + ((int64_t)b * Hq + hh) * D
                       : k_cache + (((int64_t)b * Hkv + hh) * L + pos) * D;
#pragma unroll
    for (int e = 0; e < E; ++e) dst[lane * E + e] = from_f32<T>(o[e]);
}

// -------------------------------------------------------- decode attention
// The keys 0..pos of one (row b, kv head g) are split over S CTAs
// (flash-decoding): CTA (b, g, s) takes keys [s*c, min((s+1)*c, n)),
// c = ceil(n / S), and computes, for the G query heads that share kv head g,
// the chunk's maximum score m, the sum l of exp(score - m) and the
// unnormalised sum acc of exp(score - m) * v.  With S = 1 it writes
// acc / l; otherwise it writes (m, l, acc) to the workspace and the CTA that
// arrives last for (b, g) combines the S chunks in chunk order, rescaling each
// by exp(m_s - M), and resets the arrival counter.  D threads per CTA; keys
// are read in batches of 8 per warp with independent loads (the cache reads
// are latency-bound at decode sizes); softmax and the weighted sum of values
// run in fp32.
// ROPE: the CTA first normalises and rotates its G query heads (kept in
// shared memory); the CTA whose chunk holds position pos also normalises and
// rotates the kv head's new k row and writes the new k and v rows at pos to
// the caches, reading the row back after a barrier.  A position outside the
// cache gives a zero output and writes nothing.
template <typename T> struct AttnRope {
    const T *k, *v;                    // this step's k / v projections [B, Hkv, D]
    const float *qw, *kw;              // per-head norm weights [D] (may be null)
    const float *cosT, *sinT;          // [L, D]
    float eps;
};

struct AttnSplit {
    int S;                             // CTAs per (b, g)
    int cmax;                          // score slots per head in shared memory (>= ceil(n / S))
    float *part;                       // S > 1: [B * Hkv][S][G * D + 2 * G] fp32
    uint32_t *count;                   // S > 1: [B * Hkv] arrival counters (0 between launches)
    int cluster;                       // the S CTAs of a (b, g) are one thread-block cluster:
                                       // partial states combined through distributed shared memory
};

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// A float at shared address `a` (this CTA's layout) in cluster CTA `rank`.
__device__ __forceinline__ float ld_cluster_f32(uint32_t a, uint32_t rank) {
    uint32_t ra;
    float v;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(rank));
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(ra) : "memory");
    return v;
}

template <typename T, int D, int G, bool ROPE>
__global__ void __launch_bounds__(D) k_attn_decode(const T *q, T *k_cache, T *v_cache,
                                                   const int64_t *pos_dev, int Hq, int Hkv, int64_t L,
                                                   float scale, T *out, const AttnRope<T> rp,
                                                   const AttnSplit sp) {
    constexpr int NW = D / 32, E = D / 32, KB = 8;
    extern __shared__ float sc[];                 // scores [G][cmax]
    __shared__ float red[G][NW];
    __shared__ float stat[G][2];                  // max, sum
    __shared__ float qs[ROPE ? G : 1][D];         // ROPE: the rotated queries
    __shared__ int last;
    pdl_launch_dependents();
    const int S = sp.S, cmax = sp.cmax;
    const int bg = blockIdx.x / S, s = blockIdx.x - (blockIdx.x / S) * S;
    const int b = bg / Hkv, g = bg - b * Hkv;
    if (threadIdx.x == 0) {
        // Before waiting for the kernel that wrote q/k/v: start the cache rows
        // of the earlier positions on their way into L2 (a hint only: the
        // position read here may be stale, the range is clamped to the cache).
        const int64_t p0 = min(max(*(volatile const int64_t *)pos_dev, (int64_t)0), L);
        const int64_t c0 = (p0 + 1 + S - 1) / S;
        const int64_t a0 = min((int64_t)s * c0, p0), a1 = min(a0 + c0, p0);
        if (a1 > a0) {
            const uint32_t bytes = (uint32_t)((a1 - a0) * D * sizeof(T));
            const int64_t off = ((int64_t)bg * L + a0) * D;
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(k_cache + off), "r"(bytes) : "memory");
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(v_cache + off), "r"(bytes) : "memory");
        }
    }
    pdl_wait();
    const int64_t pos = *pos_dev;
    int64_t n = min(pos + 1, L);                       // keys 0..pos (none if pos < 0)
    if (ROPE && pos >= L) n = 0;
    const int64_t c = n > 0 ? (n + S - 1) / S : 0;
    const int64_t j0c = min((int64_t)s * c, n), j1c = min(j0c + c, n);
    const int64_t nc = j1c - j0c;                       // this chunk's keys
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (ROPE) {
        if (nc > 0) {
            // warp w takes heads w, w + NW, ... of the G query heads, and (the
            // chunk holding pos only) k and v; all its loads (and the
            // position's cos / sin) are issued first
            const bool own = pos >= j0c && pos < j1c;
            const int items = own ? G + 2 : G;
            constexpr int R = (G + 2 + NW - 1) / NW;
            const T *kp = rp.k, *vp = rp.v;
            const float *qw = rp.qw, *kw = rp.kw;
            float xs[R][E], cs[E], sn[E];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int hh = warp + NW * r;
                if (hh < items) {
                    const T *src = hh < G ? q + ((int64_t)b * Hq + g * G + hh) * D
                                          : (hh == G ? kp : vp) + ((int64_t)b * Hkv + g) * D;
#pragma unroll
                    for (int e = 0; e < E; ++e) xs[r][e] = ld(src, lane * E + e);
                }
            }
            rope_row<T, E>(rp.cosT + pos * D, rp.sinT + pos * D, lane, cs, sn);
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int hh = warp + NW * r;
                if (hh >= items) break;
                if (hh == G + 1) {
                    T *dst = v_cache + (((int64_t)b * Hkv + g) * L + pos) * D;
#pragma unroll
                    for (int e = 0; e < E; ++e) dst[lane * E + e] = from_f32<T>(xs[r][e]);
                    continue;
                }
                float o[E];
                qk_head<T, E>(xs[r], rp.eps, hh < G ? qw : kw, cs, sn, lane, o);
                if (hh < G) {
#pragma unroll
                    for (int e = 0; e < E; ++e) qs[hh][lane * E + e] = o[e];
                } else {
                    T *dst = k_cache + (((int64_t)b * Hkv + g) * L + pos) * D;
#pragma unroll
                    for (int e = 0; e < E; ++e) dst[lane * E + e] = from_f32<T>(o[e]);
                }
            }
        }
        __syncthreads();                              // rotated queries and the new cache row
    }
    float qv[G][E];
#pragma unroll
    for (int h = 0; h < G; ++h) {
        const T *qr = q + ((int64_t)b * Hq + g * G + h) * D;
#pragma unroll
        for (int e = 0; e < E; ++e) qv[h][e] = ROPE ? qs[h][lane * E + e] : ld(qr, lane * E + e);
    }
    const T *kb = k_cache + ((int64_t)b * Hkv + g) * L * D;     // same pointer as the writes above
    const T *vb = v_cache + ((int64_t)b * Hkv + g) * L * D;
    float mx[G];
#pragma unroll
    for (int h = 0; h < G; ++h) mx[h] = -INFINITY;
    for (int64_t u0 = (int64_t)warp * KB; u0 < nc; u0 += (int64_t)NW * KB) {
        float kv[KB][E];
#pragma unroll
        for (int u = 0; u < KB; ++u) {                // KB independent row loads
            const int64_t j = j0c + min(u0 + u, nc - 1);
#pragma unroll
            for (int e = 0; e < E; ++e) kv[u][e] = ld(kb, j * D + lane * E + e);
        }
#pragma unroll
        for (int u = 0; u < KB; ++u) {
#pragma unroll
            for (int h = 0; h < G; ++h) {
                float d = 0.f;
#pragma unroll
                for (int e = 0; e < E; ++e) d += qv[h][e] * kv[u][e];
                d = warp_sum(d) * scale;
                if (u0 + u < nc) {
                    if (lane == 0) sc[h * cmax + u0 + u] = d;
                    mx[h] = fmaxf(mx[h], d);
                }
            }
        }
    }
#pragma unroll
    for (int h = 0; h < G; ++h)
        if (lane == 0) red[h][warp] = mx[h];
    __syncthreads();
    if (threadIdx.x < G) {
        float m = -INFINITY;
        for (int w = 0; w < NW; ++w) m = fmaxf(m, red[threadIdx.x][w]);
        stat[threadIdx.x][0] = m;
    }
    __syncthreads();
    float sum[G];
#pragma unroll
    for (int h = 0; h < G; ++h) {
        sum[h] = 0.f;
        const float m = stat[h][0];
        for (int64_t j = threadIdx.x; j < nc; j += D) {
            const float p = expf(sc[h * cmax + j] - m);
            sc[h * cmax + j] = p;
            sum[h] += p;
        }
        sum[h] = warp_sum(sum[h]);
    }
    __syncthreads();                                  // red[] reuse; sc[] published below
#pragma unroll
    for (int h = 0; h < G; ++h)
        if (lane == 0) red[h][warp] = sum[h];
    __syncthreads();
    if (threadIdx.x < G) {
        float t = 0.f;
        for (int w = 0; w < NW; ++w) t += red[threadIdx.x][w];
        stat[threadIdx.x][1] = t;
    }
    __syncthreads();
    // acc[h][i] = sum_j p_h[j] v[j][i]: thread i, KB independent value loads per step
    const int i = threadIdx.x;
    float acc[G];
#pragma unroll
    for (int h = 0; h < G; ++h) acc[h] = 0.f;
    int64_t j = 0;
    for (; j + KB <= nc; j += KB) {
        float vv[KB];
#pragma unroll
        for (int u = 0; u < KB; ++u) vv[u] = ld(vb, (j0c + j + u) * D + i);
#pragma unroll
        for (int u = 0; u < KB; ++u)
#pragma unroll
            for (int h = 0; h < G; ++h) acc[h] = fmaf(sc[h * cmax + j + u], vv[u], acc[h]);
    }
    for (; j < nc; ++j) {
        const float v = ld(vb, (j0c + j) * D + i);
#pragma unroll
        for (int h = 0; h < G; ++h) acc[h] = fmaf(sc[h * cmax + j], v, acc[h]);
    }
    T *ob = out + ((int64_t)b * Hq + g * G) * D;
    if (S == 1) {
#pragma unroll
        for (int h = 0; h < G; ++h) ob[h * D + i] = from_f32<T>(n > 0 ? acc[h] / stat[h][1] : 0.f);
        return;
    }
    constexpr int PW = G * D + 2 * G;
    if (sp.cluster) {
        // this chunk's (m, l, acc) in shared memory; after a cluster barrier
        // CTA s of the (b, g) cluster combines outputs [s * per, (s + 1) * per)
        // of the G * D from every chunk's state (chunk order, the arithmetic of
        // the workspace combine below), then a second barrier keeps every
        // CTA's state alive until all have read it
        __shared__ float cst[PW];
#pragma unroll
        for (int h = 0; h < G; ++h) cst[h * D + i] = acc[h];
        if (i < G) {
            cst[G * D + i] = nc > 0 ? stat[i][0] : -INFINITY;
            cst[G * D + G + i] = nc > 0 ? stat[i][1] : 0.f;
        }
        cluster_sync_all();
        const uint32_t cb = smem_u32(cst);
        const int per = (G * D + S - 1) / S;
        const int e1 = min((s + 1) * per, G * D);
        for (int e = s * per + (int)threadIdx.x; e < e1; e += D) {
            const int h = e / D;
            float M = -INFINITY;
            for (int t = 0; t < S; ++t) M = fmaxf(M, ld_cluster_f32(cb + 4u * (G * D + h), (uint32_t)t));
            float lsum = 0.f, o = 0.f;
            for (int t = 0; t < S; ++t) {
                const float mt = ld_cluster_f32(cb + 4u * (G * D + h), (uint32_t)t);
                const float f = mt == -INFINITY ? 0.f : expf(mt - M);
                lsum = fmaf(ld_cluster_f32(cb + 4u * (G * D + G + h), (uint32_t)t), f, lsum);
                o = fmaf(ld_cluster_f32(cb + 4u * e, (uint32_t)t), f, o);
            }
            ob[e] = from_f32<T>(lsum > 0.f ? o / lsum : 0.f);
        }
        cluster_sync_all();
        return;
    }
    // this chunk's (m, l, acc) -> the workspace; the last CTA of (b, g) combines
    float *pp = sp.part + ((int64_t)bg * S + s) * PW;
#pragma unroll
    for (int h = 0; h < G; ++h) pp[h * D + i] = acc[h];
    if (i < G) {
        pp[G * D + i] = nc > 0 ? stat[i][0] : -INFINITY;
        pp[G * D + G + i] = nc > 0 ? stat[i][1] : 0.f;
    }
    __threadfence();                                  // the chunk's values before its arrival
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(sp.count + bg, 1u) == (uint32_t)(S - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    // combine: every chunk's (m, l) into shared memory with independent loads,
    // then per head M = max m_s, L = sum_s l_s exp(m_s - M) and the weight
    // f_s = exp(m_s - M) / L of each chunk (chunk order), then thread i adds
    // its dimension of the S chunks' acc with all loads issued first
    const float *pb = sp.part + (int64_t)bg * S * PW;
    float *fw = sc;                                   // [S][G] chunk weights (the scores are consumed)
    for (int e = threadIdx.x; e < S * G; e += D) {
        const int t = e / G, h = e - (e / G) * G;
        fw[e] = __ldcg(pb + (int64_t)t * PW + G * D + h);
        fw[S * G + e] = __ldcg(pb + (int64_t)t * PW + G * D + G + h);
    }
    __syncthreads();
    if (threadIdx.x < G) {
        const int h = threadIdx.x;
        float M = -INFINITY;
        for (int t = 0; t < S; ++t) M = fmaxf(M, fw[t * G + h]);
        float lsum = 0.f;
        for (int t = 0; t < S; ++t) {
            const float mt = fw[t * G + h];
            const float f = mt == -INFINITY ? 0.f : expf(mt - M);
            fw[2 * S * G + t * G + h] = f;
            lsum = fmaf(fw[S * G + t * G + h], f, lsum);
        }
        stat[h][1] = lsum;
    }
    __syncthreads();
    float o[G];
#pragma unroll
    for (int h = 0; h < G; ++h) o[h] = 0.f;
    constexpr int CB = 8;                             // chunks whose loads are issued together
    for (int t0 = 0; t0 < S; t0 += CB) {
        float av[CB][G];
#pragma unroll
        for (int u = 0; u < CB; ++u)
#pragma unroll
            for (int h = 0; h < G; ++h)
                av[u][h] = t0 + u < S ? __ldcg(pb + (int64_t)(t0 + u) * PW + h * D + i) : 0.f;
#pragma unroll
        for (int u = 0; u < CB; ++u)
#pragma unroll
            for (int h = 0; h < G; ++h)
                if (t0 + u < S) o[h] = fmaf(av[u][h], fw[2 * S * G + (t0 + u) * G + h], o[h]);
    }
#pragma unroll
    for (int h = 0; h < G; ++h) {
        const float lsum = stat[h][1];
        ob[h * D + i] = from_f32<T>(lsum > 0.f ? o[h] / lsum : 0.f);
    }
    if (threadIdx.x == 0) sp.count[bg] = 0u;          // ready for the next launch
}

// ------------------------------------------------------------- greedy pick
// next_ids[b] = argmax over the vocabulary of logits row b, the vocabulary
// split over `world` ranks (this rank holds ids [rank*V, (rank+1)*V)).  One
// CTA per row: thread-level then warp-level (max, lowest index on ties), then
// for world > 1 thread 0 stores (value, global id) as two epoch-flagged
// 64-bit words into slot `rank` of every rank's pick buffer (peer memory) and
// reads every rank's pair from its own buffer (bounded wait for the epoch);
// the largest value wins, the lowest rank on ties (= the lowest id, torch's
// first-index rule).
__device__ __forceinline__ void st_sys_u64(uint64_t *p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_sys_u64(const uint64_t *p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

struct PickPeers {
    uint64_t *slot[8];                 // rank p's pick buffer, this rank's slot ([B][2] words)
};

__device__ __forceinline__ bool pick_better(float v, int64_t i, float bv, int64_t bi) {
    return v > bv || (v == bv && i < bi) || (bv != bv && v == v);
}

template <typename T>
__global__ void __launch_bounds__(1024) k_greedy_pick(const T *logits, int64_t V, int64_t ld, int rank, int world,
                                                     const PickPeers pp, const uint64_t *local, const uint32_t *epoch,
                                                     int64_t *next_ids, uint32_t *status) {
    __shared__ float sv[32];
    __shared__ int64_t si[32];
    pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const T *row = logits + (int64_t)b * ld;
    float bv = -INFINITY;
    int64_t bi = INT64_MAX;
    for (int64_t i = tid; i < V; i += blockDim.x) {
        const float v = to_f32<T>(row[i]);
        if (pick_better(v, i, bv, bi)) { bv = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float v = __shfl_xor_sync(0xffffffffu, bv, o);
        const int64_t i = __shfl_xor_sync(0xffffffffu, bi, o);
        if (pick_better(v, i, bv, bi)) { bv = v; bi = i; }
    }
    if (lane == 0) { sv[w] = bv; si[w] = bi; }
    __syncthreads();
    if (tid != 0) return;
    bv = sv[0]; bi = si[0];
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i)
        if (pick_better(sv[i], si[i], bv, bi)) { bv = sv[i]; bi = si[i]; }
    int64_t id = bi + (int64_t)rank * V;
    if (world > 1) {
        const uint64_t ep = (uint64_t)*epoch << 32;
        for (int p = 0; p < world; ++p) {
            st_sys_u64(pp.slot[p] + 2 * b, ep | __float_as_uint(bv));
            st_sys_u64(pp.slot[p] + 2 * b + 1, ep | (uint32_t)id);
        }
        float gv = -INFINITY;
        int64_t gid = INT64_MAX;
        const uint64_t t0 = global_timer_ns();
        for (int p = 0; p < world; ++p) {
            const uint64_t *q = local + ((int64_t)p * gridDim.x + b) * 2;
            uint64_t a, c;
            while (true) {
                a = ld_sys_u64(q);
                c = ld_sys_u64(q + 1);
                if ((a >> 32) == (ep >> 32) && (c >> 32) == (ep >> 32)) break;
                if (global_timer_ns() - t0 > kWaitNs) {
                    report(status, CBQ_FLAG_TIMEOUT, (uint32_t)b);
                    return;                                // next_ids[b] keeps its old value
                }
                __nanosleep(32);
            }
            const float v = __uint_as_float((uint32_t)a);
            const int64_t i = (int64_t)(uint32_t)c;
            if (pick_better(v, i, gv, gid)) { gv = v; gid = i; }
        }
        id = gid;
    }
    next_ids[b] = id;
}

// out[i] = round(round(silu(g[i])) * u[i]) (g, u already rounded to T): the
// SiLU * up of a transformer MLP when gate and up were computed separately,
// with the rounding of the torch sequence (and of the GEMV epilogue).
template <typename T>
__global__ void __launch_bounds__(256) k_silu_mul(const T *g, const T *u, int64_t n, T *out) {
    pdl_launch_dependents();
    pdl_wait();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float gv = to_f32<T>(g[i]), uv = to_f32<T>(u[i]);
        const float sv = to_f32<T>(from_f32<T>(gv / (1.0f + expf(-gv))));
        out[i] = from_f32<T>(sv * uv);
    }
}

}  // namespace

// ------------------------------------------------------------------- C ABI

extern "C" int cbq_greedy_pick(const void *logits_dev, int dtype, int64_t B, int64_t V, int64_t ld, int rank,
                               int world, void *const *slot_dev, const void *local_slots_dev,
                               const uint32_t *epoch_dev, int64_t *next_ids_dev, uint32_t *status_dev,
                               void *stream) {
    if (B < 0 || V < 1 || ld < V || world < 1 || world > 8 || rank < 0 || rank >= world ||
        (dtype != CBQ_F32 && dtype != CBQ_BF16))
        return CBQ_ERR_ARG;
    if (B == 0) return CBQ_OK;
    if (!logits_dev || !next_ids_dev || B > 65535 || (int64_t)V * world >= (1ll << 32)) return CBQ_ERR_ARG;
    PickPeers pp{};
    if (world > 1) {
        if (!slot_dev || !local_slots_dev || !epoch_dev) return CBQ_ERR_ARG;
        for (int p = 0; p < world; ++p) {
            if (!slot_dev[p] || (reinterpret_cast<uintptr_t>(slot_dev[p]) & 7)) return CBQ_ERR_ARG;
            pp.slot[p] = static_cast<uint64_t *>(slot_dev[p]);
        }
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (dtype == CBQ_F32)
        CBQ_CUDA_TRY(cbq_host::launch_pdl(k_greedy_pick<float>, dim3((unsigned)B), dim3(1024), 0, s,
                                          static_cast<const float *>(logits_dev), V, ld, rank, world, pp,
                                          static_cast<const uint64_t *>(local_slots_dev), epoch_dev, next_ids_dev,
                                          status_dev));
    else
        CBQ_CUDA_TRY(cbq_host::launch_pdl(k_greedy_pick<__nv_bfloat16>, dim3((unsigned)B), dim3(1024), 0, s,
                                          static_cast<const __nv_bfloat16 *>(logits_dev), V, ld, rank, world, pp,
                                          static_cast<const uint64_t *>(local_slots_dev), epoch_dev, next_ids_dev,
                                          status_dev));
    return CBQ_OK;
}

extern "C" int cbq_rmsnorm(void *x_dev, const void *add_dev, int dtype, int64_t rows, int64_t n,
                           const float *weight_dev, float eps, void *out_dev, void *stream) {
    if (rows < 0 || n < 1 || (dtype != CBQ_F32 && dtype != CBQ_BF16)) return CBQ_ERR_ARG;
    if (rows == 0) return CBQ_OK;
    if (!x_dev || !out_dev || rows > 0x7fffffff) return CBQ_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (dtype == CBQ_F32)
        CBQ_CUDA_TRY(cbq_host::launch_pdl(k_rmsnorm<float, 256>, dim3((unsigned)rows), dim3(256), 0, s,
                                          static_cast<float *>(x_dev), static_cast<const float *>(add_dev), n,
                                          weight_dev, eps, static_cast<float *>(out_dev)));
    else
        CBQ_CUDA_TRY(cbq_host::launch_pdl(k_rmsnorm<__nv_bfloat16, 256>, dim3((unsigned)rows), dim3(256), 0, s,
                                          static_cast<__nv_bfloat16 *>(x_dev),
                                          static_cast<const __nv_bfloat16 *>(add_dev), n, weight_dev, eps,
                                          static_cast<__nv_bfloat16 *>(out_dev)));
    return CBQ_OK;
}

extern "C" int cbq_rmsnorm_allreduce(void *x_dev, const void *slots_dev, const uint32_t *counts_dev,
                                     const uint32_t *epoch_dev, int64_t expect, int world, int dtype, int64_t rows,
                                     int64_t n, const float *weight_dev, float eps, void *out_dev,
                                     uint32_t *status_dev, void *stream) {
    if (rows < 0 || n < 1 || world < 1 || world > 32 || expect < 1 || expect > 0xffffffffll ||
        (dtype != CBQ_F32 && dtype != CBQ_BF16))
        return CBQ_ERR_ARG;
    if (rows == 0) return CBQ_OK;
    if (!x_dev || !slots_dev || !counts_dev || !epoch_dev || !out_dev || rows > 0x7fffffff) return CBQ_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (dtype == CBQ_F32)
        CBQ_CUDA_TRY(cbq_host::launch_pdl(k_rmsnorm_allreduce<float, 256>, dim3((unsigned)rows), dim3(256), 0, s,
                                          static_cast<float *>(x_dev), static_cast<const float *>(slots_dev),
                                          counts_dev, epoch_dev, (uint32_t)expect, world, rows, n, weight_dev,
                                          eps, static_cast<float *>(out_dev), status_dev));
    else
        CBQ_CUDA_TRY(cbq_host::launch_pdl(k_rmsnorm_allreduce<__nv_bfloat16, 256>, dim3((unsigned)rows), dim3(256),
                                          0, s, static_cast<__nv_bfloat16 *>(x_dev),
                                          static_cast<const __nv_bfloat16 *>(slots_dev), counts_dev, epoch_dev,
                                          (uint32_t)expect, world, rows, n, weight_dev, eps,
                                          static_cast<__nv_bfloat16 *>(out_dev), status_dev));
    return CBQ_OK;
}

extern "C" int cbq_qk_norm_rope(const void *q_dev, const void *k_dev, const void *v_dev, int dtype, int64_t B,
                                int64_t Hq, int64_t Hkv, int64_t head_dim, float eps, const float *q_weight_dev,
                                const float *k_weight_dev, const float *cos_dev, const float *sin_dev,
                                const int64_t *pos_dev, void *q_out_dev, void *k_cache_dev, void *v_cache_dev,
                                int64_t cache_len, void *stream) {
    if (B < 0 || Hq < 1 || Hkv < 1 || Hq % Hkv || (dtype != CBQ_F32 && dtype != CBQ_BF16)) return CBQ_ERR_ARG;
    if (head_dim != 64 && head_dim != 128 && head_dim != 256) return CBQ_ERR_UNSUPPORTED;
    if (B == 0) return CBQ_OK;
    if (!q_dev || !k_dev || !v_dev || !cos_dev || !sin_dev || !pos_dev || !q_out_dev || !k_cache_dev ||
        !v_cache_dev || cache_len < 1)
        return CBQ_ERR_ARG;
    const int64_t warps = B * (Hq + 2 * Hkv);
    if (warps * 32 > 0x7fffffffll) return CBQ_ERR_ARG;
    const unsigned grid = (unsigned)((warps * 32 + 255) / 256);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
#define CBQ_QK(T, E)                                                                               \
    CBQ_CUDA_TRY(cbq_host::launch_pdl(                                                             \
        k_qk_norm_rope<T, E>, dim3(grid), dim3(256), 0, s, static_cast<const T *>(q_dev),           \
        static_cast<const T *>(k_dev), static_cast<const T *>(v_dev), (int)B, (int)Hq, (int)Hkv, eps, \
        q_weight_dev, k_weight_dev, cos_dev, sin_dev, pos_dev, static_cast<T *>(q_out_dev),          \
        static_cast<T *>(k_cache_dev), static_cast<T *>(v_cache_dev), cache_len))
    if (dtype == CBQ_F32) {
        if (head_dim == 64) CBQ_QK(float, 2); else if (head_dim == 128) CBQ_QK(float, 4); else CBQ_QK(float, 8);
    } else {
        if (head_dim == 64) CBQ_QK(__nv_bfloat16, 2);
        else if (head_dim == 128) CBQ_QK(__nv_bfloat16, 4);
        else CBQ_QK(__nv_bfloat16, 8);
    }
#undef CBQ_QK
    CBQ_CUDA_TRY(cudaGetLastError());
    return CBQ_OK;
}

namespace {

// Splits of the keys per (row, kv head): enough CTAs to cover the SMs about
// twice, at least 16 keys per split (cache_len bounds the keys), at most 64.
int attn_splits(int64_t B, int64_t Hkv, int64_t cache_len) {
    const int64_t target = 2 * (int64_t)cbq_host::sm_count();
    int64_t S = (target + B * Hkv - 1) / (B * Hkv);
    S = std::min<int64_t>(S, (cache_len + 15) / 16);
    S = std::min<int64_t>(S, 64);
    return (int)std::max<int64_t>(S, 1);
}

int64_t attn_workspace_bytes(int64_t B, int64_t Hkv, int64_t G, int64_t D, int S) {
    if (S <= 1) return 0;
    const int64_t part = B * Hkv * S * (G * D + 2 * G) * 4;
    return cbq_host::align_up(part, 256) + cbq_host::align_up(B * Hkv * 4, 256);
}

template <bool ROPE>
int launch_attn(const void *q_dev, void *k_cache_dev, void *v_cache_dev, int dtype, int64_t B, int64_t Hq,
                int64_t Hkv, int64_t head_dim, int64_t cache_len, const int64_t *pos_dev, float scale,
                void *out_dev, const void *k_dev, const void *v_dev, const float *qw, const float *kw,
                const float *cos_dev, const float *sin_dev, float eps, void *ws, int64_t ws_bytes,
                void *stream) {
    if (B < 0 || Hq < 1 || Hkv < 1 || Hq % Hkv || cache_len < 1 || (dtype != CBQ_F32 && dtype != CBQ_BF16))
        return CBQ_ERR_ARG;
    if (head_dim != 64 && head_dim != 128 && head_dim != 256) return CBQ_ERR_UNSUPPORTED;
    const int64_t G = Hq / Hkv;
    if (G < 1 || G > 8) return CBQ_ERR_UNSUPPORTED;
    if (B == 0) return CBQ_OK;
    if (!q_dev || !k_cache_dev || !v_cache_dev || !pos_dev || !out_dev || B * Hkv > 0x7fffffff) return CBQ_ERR_ARG;
    if (ROPE && (!k_dev || !v_dev || !cos_dev || !sin_dev)) return CBQ_ERR_ARG;
    // keys split over S CTAs when a workspace is given, else one CTA per (row, kv head)
    int S = ws ? attn_splits(B, Hkv, cache_len) : 1;
    if (ws && ws_bytes < attn_workspace_bytes(B, Hkv, G, head_dim, S)) return CBQ_ERR_ARG;
    if (B * Hkv * S > 0x7fffffff) return CBQ_ERR_ARG;
    AttnSplit sp{S, (int)((cache_len + S - 1) / S), nullptr, nullptr, 0};
    if (S > 1) {
        sp.part = static_cast<float *>(ws);
        sp.count = reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(ws) +
                                                cbq_host::align_up(B * Hkv * S * (G * head_dim + 2 * G) * 4, 256));
    }
    // scores of the group's heads; the combining CTA reuses it for 3 * S * G chunk values
    const size_t smem = std::max((size_t)sp.cmax * 4 * (size_t)G, (size_t)(S > 1 ? 3 * S * G * 4 : 0));
    if (smem > (size_t)cbq_host::max_smem_optin() - 4096 - (size_t)(G * head_dim + 2 * G) * 4 -
                   (ROPE ? (size_t)G * head_dim * 4 : 0))
        return CBQ_ERR_UNSUPPORTED;
    // up to 16 chunks: the chunks of a (row, kv head) form one thread-block
    // cluster and combine through distributed shared memory (no workspace
    // round trip); a launch the device refuses falls back to the workspace
    const bool try_cluster = S >= 2 && S <= 16 && cbq_host::attn_cluster_enabled();
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const dim3 grid((unsigned)(B * Hkv * S));
#define CBQ_AT(T, D, GG)                                                                             \
    do {                                                                                             \
        auto kern = k_attn_decode<T, D, GG, ROPE>;                                                   \
        if (smem > 32 * 1024)                                                                        \
            CBQ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
        const AttnRope<T> rp{static_cast<const T *>(k_dev), static_cast<const T *>(v_dev), qw, kw,  \
                             cos_dev, sin_dev, eps};                                                 \
        bool done = false;                                                                           \
        if (try_cluster && (S <= 8 || cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, \
                                                           1) == cudaSuccess)) {                     \
            AttnSplit spc = sp;                                                                      \
            spc.cluster = 1;                                                                         \
            done = cbq_host::launch_pdl_cluster(kern, grid, dim3(D), smem, (unsigned)S, s,           \
                                                static_cast<const T *>(q_dev), static_cast<T *>(k_cache_dev), \
                                                static_cast<T *>(v_cache_dev), pos_dev, (int)Hq, (int)Hkv, \
                                                cache_len, scale, static_cast<T *>(out_dev), rp, spc) == \
                   cudaSuccess;                                                                      \
            if (!done) (void)cudaGetLastError();                                                     \
        }                                                                                            \
        if (!done)                                                                                   \
            CBQ_CUDA_TRY(cbq_host::launch_pdl(kern, grid, dim3(D), smem, s, static_cast<const T *>(q_dev), \
                                              static_cast<T *>(k_cache_dev), static_cast<T *>(v_cache_dev), \
                                              pos_dev, (int)Hq, (int)Hkv, cache_len, scale,          \
                                              static_cast<T *>(out_dev), rp, sp));                   \
    } while (0)
#define CBQ_AT_G(T, D)                                                                               \
    do {                                                                                             \
        switch (G) {                                                                                 \
            case 1: CBQ_AT(T, D, 1); break;                                                          \
            case 2: CBQ_AT(T, D, 2); break;                                                          \
            case 3: CBQ_AT(T, D, 3); break;                                                          \
            case 4: CBQ_AT(T, D, 4); break;                                                          \
            case 5: CBQ_AT(T, D, 5); break;                                                          \
            case 6: CBQ_AT(T, D, 6); break;                                                          \
            case 7: CBQ_AT(T, D, 7); break;                                                          \
            default: CBQ_AT(T, D, 8); break;                                                         \
        }                                                                                            \
    } while (0)
    if (dtype == CBQ_F32) {
        if (head_dim == 64) CBQ_AT_G(float, 64); else if (head_dim == 128) CBQ_AT_G(float, 128);
        else CBQ_AT_G(float, 256);
    } else {
        if (head_dim == 64) CBQ_AT_G(__nv_bfloat16, 64);
        else if (head_dim == 128) CBQ_AT_G(__nv_bfloat16, 128);
        else CBQ_AT_G(__nv_bfloat16, 256);
    }
#undef CBQ_AT_G
#undef CBQ_AT
    CBQ_CUDA_TRY(cudaGetLastError());
    return CBQ_OK;
}

}  // namespace

extern "C" int cbq_attn_decode(const void *q_dev, const void *k_cache_dev, const void *v_cache_dev, int dtype,
                               int64_t B, int64_t Hq, int64_t Hkv, int64_t head_dim, int64_t cache_len,
                               const int64_t *pos_dev, float scale, void *out_dev, void *stream) {
    // the kernel only reads the cache in this form
    return launch_attn<false>(q_dev, const_cast<void *>(k_cache_dev), const_cast<void *>(v_cache_dev), dtype, B,
                              Hq, Hkv, head_dim, cache_len, pos_dev, scale, out_dev, nullptr, nullptr, nullptr,
                              nullptr, nullptr, nullptr, 0.f, nullptr, 0, stream);
}

extern "C" int cbq_attn_decode_rope(const void *q_dev, const void *k_dev, const void *v_dev, int dtype, int64_t B,
                                    int64_t Hq, int64_t Hkv, int64_t head_dim, float eps,
                                    const float *q_weight_dev, const float *k_weight_dev, const float *cos_dev,
                                    const float *sin_dev, const int64_t *pos_dev, void *k_cache_dev,
                                    void *v_cache_dev, int64_t cache_len, float scale, void *out_dev,
                                    void *stream) {
    return launch_attn<true>(q_dev, k_cache_dev, v_cache_dev, dtype, B, Hq, Hkv, head_dim, cache_len, pos_dev,
                             scale, out_dev, k_dev, v_dev, q_weight_dev, k_weight_dev, cos_dev, sin_dev, eps,
                             nullptr, 0, stream);
}

extern "C" int64_t cbq_attn_workspace_bytes(int64_t B, int64_t Hq, int64_t Hkv, int64_t head_dim,
                                            int64_t cache_len) {
    if (B < 0 || Hq < 1 || Hkv < 1 || Hq % Hkv || head_dim < 1 || cache_len < 1) return -1;
    return std::max<int64_t>(attn_workspace_bytes(B, Hkv, Hq / Hkv, head_dim, attn_splits(B, Hkv, cache_len)), 256);
}

extern "C" int cbq_attn_decode_rope_split(const void *q_dev, const void *k_dev, const void *v_dev, int dtype,
                                          int64_t B, int64_t Hq, int64_t Hkv, int64_t head_dim, float eps,
                                          const float *q_weight_dev, const float *k_weight_dev,
                                          const float *cos_dev, const float *sin_dev, const int64_t *pos_dev,
                                          void *k_cache_dev, void *v_cache_dev, int64_t cache_len, float scale,
                                          void *out_dev, void *workspace_dev, int64_t workspace_bytes,
                                          void *stream) {
    if (!workspace_dev) return CBQ_ERR_ARG;
    return launch_attn<true>(q_dev, k_cache_dev, v_cache_dev, dtype, B, Hq, Hkv, head_dim, cache_len, pos_dev,
                             scale, out_dev, k_dev, v_dev, q_weight_dev, k_weight_dev, cos_dev, sin_dev, eps,
                             workspace_dev, workspace_bytes, stream);
}

extern "C" int cbq_attn_decode_split(const void *q_dev, const void *k_cache_dev, const void *v_cache_dev,
                                     int dtype, int64_t B, int64_t Hq, int64_t Hkv, int64_t head_dim,
                                     int64_t cache_len, const int64_t *pos_dev, float scale, void *out_dev,
                                     void *workspace_dev, int64_t workspace_bytes, void *stream) {
    if (!workspace_dev) return CBQ_ERR_ARG;
    return launch_attn<false>(q_dev, const_cast<void *>(k_cache_dev), const_cast<void *>(v_cache_dev), dtype, B,
                              Hq, Hkv, head_dim, cache_len, pos_dev, scale, out_dev, nullptr, nullptr, nullptr,
                              nullptr, nullptr, nullptr, 0.f, workspace_dev, workspace_bytes, stream);
}

extern "C" int cbq_silu_mul(const void *g_dev, const void *u_dev, int dtype, int64_t n, void *out_dev,
                            void *stream) {
    if (n < 0 || (dtype != CBQ_F32 && dtype != CBQ_BF16)) return CBQ_ERR_ARG;
    if (n == 0) return CBQ_OK;
    if (!g_dev || !u_dev || !out_dev) return CBQ_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const unsigned blocks = (unsigned)std::min<int64_t>((n + 255) / 256, (int64_t)cbq_host::sm_count() * 4);
    if (dtype == CBQ_F32)
        CBQ_CUDA_TRY(cbq_host::launch_pdl(k_silu_mul<float>, dim3(blocks), dim3(256), 0, s,
                                          static_cast<const float *>(g_dev), static_cast<const float *>(u_dev), n,
                                          static_cast<float *>(out_dev)));
    else
        CBQ_CUDA_TRY(cbq_host::launch_pdl(k_silu_mul<__nv_bfloat16>, dim3(blocks), dim3(256), 0, s,
                                          static_cast<const __nv_bfloat16 *>(g_dev),
                                          static_cast<const __nv_bfloat16 *>(u_dev), n,
                                          static_cast<__nv_bfloat16 *>(out_dev)));
    return CBQ_OK;
}
