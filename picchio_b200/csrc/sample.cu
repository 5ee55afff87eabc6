// sample.cu - sample_logits (picchio.c:1540-1649) as one block-wide kernel.
//
// The reference's sampler is a chain of sequential fp32 passes over the
// vocabulary.  Everything that does not depend on evaluation order runs in
// parallel here: the penalty (each id's divisions in sequence, ids
// independent), the temperature multiply, the top-k threshold (an exact
// radix select of the k-th largest value instead of a full sort), the max,
// the exponentials and the normalising divisions.  Every fp32 SUM keeps the
// reference's order: the nonzero terms are compacted in index order and one
// thread adds them in sequence (adding the zeros the reference also adds
// changes nothing), so the sums, the top-p cut and the final cumulative draw
// see the same values.  expf is evaluated as the correctly rounded double
// exponential rounded to fp32.  Top-p candidates are sorted inside the block
// when they fit (SAMPLE_SORT_CAP), else by a stable device radix sort between
// two launches; ties are ordered by token id.
#include "sample.h"

#include <cub/device/device_radix_sort.cuh>

#include <climits>

#include "launch.cuh"

namespace pc {
namespace {

constexpr int ST = 1024;        // threads of the sampler block
constexpr int NW = ST / 32;
constexpr int CH = 4096;        // staging chunk of the sequential passes
constexpr unsigned FULL = 0xffffffffu;

struct SampleSmem {
    union {
        int owners[SAMPLE_HIST_CAP];
        struct {
            float key[SAMPLE_SORT_CAP];
            int pos[SAMPLE_SORT_CAP];
        } cand;
        float stage[CH];
    } u;
    int hist[2048];
    float rf[NW];
    int ri[NW];
    int rj[NW];
    int n_owner;
    int bi[4];
    float bf[4];
};

struct SampleArgs {
    const float *logits;
    int V;
    int big;
    SampleState *s;
    int *hist;
    int *cnt;
    float *w;
    float *nz_val;
    int *nz_idx;
    float *ck;
    int *cv;
    const float *sk;
    const int *sv;
    int *ids;
    int *ids2;
    int *err;
};

__device__ __forceinline__ uint32_t fkey(float f) {  // order-preserving float -> uint
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float fkey_inv(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k ^ 0x80000000u) : ~k);
}

__device__ float block_max(float v, SampleSmem &sm) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float t = __shfl_xor_sync(FULL, v, o);
        v = t > v ? t : v;
    }
    if (lane == 0) sm.rf[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = sm.rf[lane];
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float t = __shfl_xor_sync(FULL, v, o);
            v = t > v ? t : v;
        }
        if (lane == 0) sm.bf[0] = v;
    }
    __syncthreads();
    v = sm.bf[0];
    __syncthreads();
    return v;
}

__device__ int block_sum_i(int v, SampleSmem &sm) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    if (lane == 0) sm.ri[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = sm.ri[lane];
#pragma unroll
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
        if (lane == 0) sm.bi[0] = v;
    }
    __syncthreads();
    v = sm.bi[0];
    __syncthreads();
    return v;
}

__device__ int block_max_i(int v, SampleSmem &sm) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) v = max(v, __shfl_xor_sync(FULL, v, o));
    if (lane == 0) sm.ri[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = sm.ri[lane];
#pragma unroll
        for (int o = 16; o; o >>= 1) v = max(v, __shfl_xor_sync(FULL, v, o));
        if (lane == 0) sm.bi[0] = v;
    }
    __syncthreads();
    v = sm.bi[0];
    __syncthreads();
    return v;
}

// Exclusive prefix sum of v over the block (thread order); *total = the sum.
__device__ int block_excl_scan(int v, int *total, SampleSmem &sm) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(FULL, incl, o);
        if (lane >= o) incl += t;
    }
    if (lane == 31) sm.ri[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const int wv = sm.ri[lane];
        int wi = wv;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(FULL, wi, o);
            if (lane >= o) wi += t;
        }
        sm.rj[lane] = wi - wv;
        if (lane == 31) sm.bi[1] = wi;
    }
    __syncthreads();
    const int r = sm.rj[warp] + incl - v;
    *total = sm.bi[1];
    __syncthreads();
    return r;
}

// First index of the largest value (picchio.c:1557-1559: strict >, so ties
// go to the lowest index); 0 when nothing beats -inf.
__device__ int block_argmax(const float *w, int V, SampleSmem &sm) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float bv = -INFINITY;
    int bi = INT_MAX;
    for (int i = threadIdx.x; i < V; i += ST) {
        const float v = w[i];
        if (v > bv) { bv = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float tv = __shfl_xor_sync(FULL, bv, o);
        const int ti = __shfl_xor_sync(FULL, bi, o);
        if (tv > bv || (tv == bv && ti < bi)) { bv = tv; bi = ti; }
    }
    if (lane == 0) { sm.rf[warp] = bv; sm.ri[warp] = bi; }
    __syncthreads();
    if (warp == 0) {
        bv = sm.rf[lane];
        bi = sm.ri[lane];
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float tv = __shfl_xor_sync(FULL, bv, o);
            const int ti = __shfl_xor_sync(FULL, bi, o);
            if (tv > bv || (tv == bv && ti < bi)) { bv = tv; bi = ti; }
        }
        if (lane == 0) sm.bi[0] = bi == INT_MAX ? 0 : bi;
    }
    __syncthreads();
    const int r = sm.bi[0];
    __syncthreads();
    return r;
}

// The k-th largest of w[0..V) (1 <= k < V): the value the reference reads at
// position k - 1 of its descending sort (picchio.c:1575-1576), by an exact
// three-pass radix select (11 + 11 + 10 bits) on order-preserving keys.
__device__ float kth_largest(const float *w, int V, int k, SampleSmem &sm) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t prefix = 0, mask = 0;
    int krem = k;
    for (int pass = 0; pass < 3; ++pass) {
        const int sh = pass == 0 ? 21 : pass == 1 ? 10 : 0;
        const int nb = pass == 2 ? 1024 : 2048;
        for (int b = threadIdx.x; b < 2048; b += ST) sm.hist[b] = 0;
        __syncthreads();
        for (int base = 0; base < V; base += ST) {
            const int i = base + threadIdx.x;
            const uint32_t key = i < V ? fkey(w[i]) : 0u;
            const bool in = i < V && (key & mask) == prefix;
            const unsigned act = __ballot_sync(FULL, in);
            if (in) {  // one shared-memory atomic per distinct bin of the warp
                const int bin = (int)((key >> sh) & (uint32_t)(nb - 1));
                const unsigned peers = __match_any_sync(act, bin);
                if ((__ffs(peers) - 1) == lane) atomicAdd(&sm.hist[bin], __popc(peers));
            }
        }
        __syncthreads();
        if (warp == 0) {  // the bin holding the krem-th largest, scanning from the top
            const int per = nb / 32, hi = nb - lane * per;
            int s = 0;
            for (int b = hi - 1; b >= hi - per; --b) s += sm.hist[b];
            int incl = s;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int t = __shfl_up_sync(FULL, incl, o);
                if (lane >= o) incl += t;
            }
            const unsigned hit = __ballot_sync(FULL, incl >= krem);
            if (lane == __ffs(hit) - 1) {
                int above = incl - s, d = hi - per;
                for (int b = hi - 1; b >= hi - per; --b) {
                    if (above + sm.hist[b] >= krem) { d = b; break; }
                    above += sm.hist[b];
                }
                sm.bi[2] = d;
                sm.bi[3] = krem - above;
            }
        }
        __syncthreads();
        prefix |= (uint32_t)sm.bi[2] << sh;
        mask |= (uint32_t)(nb - 1) << sh;
        krem = sm.bi[3];
        __syncthreads();
    }
    return fkey_inv(prefix);
}

// v[0] + v[1] + ... + v[n-1] in fp32, in that order, starting from 0.
__device__ float seq_sum(const float *v, int n, SampleSmem &sm) {
    float s = 0.0f;
    for (int base = 0; base < n; base += CH) {
        const int m = min(CH, n - base);
        for (int i = threadIdx.x; i < m; i += ST) sm.u.stage[i] = v[base + i];
        __syncthreads();
        if (threadIdx.x == 0)
            for (int i = 0; i < m; ++i) s = __fadd_rn(s, sm.u.stage[i]);
        __syncthreads();
    }
    if (threadIdx.x == 0) sm.bf[1] = s;
    __syncthreads();
    s = sm.bf[1];
    __syncthreads();
    return s;
}

// The top-p cut (picchio.c:1610-1616): the first position at which the
// running fp32 sum of the descending probabilities reaches top_p, plus one;
// n when it never does.
__device__ int seq_cut(const float *sorted, int n, float top_p, SampleSmem &sm) {
    float cum = 0.0f;
    int cut = n;
    for (int base = 0; base < n && cut == n; base += CH) {
        const int m = min(CH, n - base);
        for (int i = threadIdx.x; i < m; i += ST) sm.u.stage[i] = sorted[base + i];
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int i = 0; i < m; ++i) {
                cum = __fadd_rn(cum, sm.u.stage[i]);
                if (cum >= top_p) { cut = base + i + 1; break; }
            }
            sm.bi[2] = cut;
        }
        __syncthreads();
        cut = sm.bi[2];
        __syncthreads();
    }
    return cut;
}

// Zeroes the candidates past the cut, renormalises (picchio.c:1618-1624).
__device__ void apply_cut(const SampleArgs &a, int n_nz, const int *pos, int cut, int n_c, SampleSmem &sm) {
    for (int j = cut + threadIdx.x; j < n_c; j += ST) a.nz_val[pos[j]] = 0.0f;
    __syncthreads();
    const float s2 = seq_sum(a.nz_val, n_nz, sm);
    if (s2 > 0.0f)
        for (int j = threadIdx.x; j < n_nz; j += ST) a.nz_val[j] = __fdiv_rn(a.nz_val[j], s2);
    __syncthreads();
}

__device__ void emit(const SampleArgs &a, int id, bool record) {
    if (threadIdx.x == 0) {
        a.ids[0] = id;
        if (a.ids2) a.ids2[0] = id;
        const int hl = a.s->hist_len;
        if (record && hl < SAMPLE_HIST_CAP) {
            a.hist[hl] = id;
            a.s->hist_len = hl + 1;
        }
    }
}

// The draw (picchio.c:1631-1647): r from the generator, the first id whose
// running sum of probabilities in index order reaches r, else the last id of
// nonzero probability, else 0 (not recorded, as in the reference).
__device__ void draw(const SampleArgs &a, int n_nz, SampleSmem &sm) {
    unsigned long long st = a.s->rng;
    st ^= st << 13;
    st ^= st >> 7;
    st ^= st << 17;
    const float r = __fdiv_rn(__ull2float_rn(st >> 33), 2147483648.0f);
    __syncthreads();
    if (threadIdx.x == 0) a.s->rng = st;
    if (!(r > 0.0f)) {  // the running sum (>= 0) reaches r at id 0
        emit(a, 0, true);
        return;
    }
    float cum = 0.0f;
    int id = -1;
    for (int base = 0; base < n_nz && id < 0; base += CH) {
        const int m = min(CH, n_nz - base);
        for (int i = threadIdx.x; i < m; i += ST) sm.u.stage[i] = a.nz_val[base + i];
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int i = 0; i < m; ++i) {
                cum = __fadd_rn(cum, sm.u.stage[i]);
                if (cum >= r) { id = a.nz_idx[base + i]; break; }
            }
            sm.bi[2] = id;
        }
        __syncthreads();
        id = sm.bi[2];
        __syncthreads();
    }
    if (id >= 0) {
        emit(a, id, true);
        return;
    }
    int last = -1;
    for (int j = threadIdx.x; j < n_nz; j += ST)
        if (a.nz_val[j] > 0.0f) last = j;
    last = block_max_i(last, sm);
    if (last >= 0) emit(a, a.nz_idx[last], true);
    else emit(a, 0, false);
}

__global__ void __launch_bounds__(ST, 1) sample_kernel(const SampleArgs a) {
    __shared__ SampleSmem sm;
    pdl_wait();
    pdl_trigger();
    SampleState *s = a.s;
    const SampleParams P = s->p;
    const int V = a.V, tid = threadIdx.x;
    const bool greedy = P.temperature < 1e-6f;
    if (tid == 0) s->stage = 0;

    // penalty (picchio.c:1542-1552) and temperature (1564-1565)
    for (int i = tid; i < V; i += ST) {
        const float v = a.logits[i];
        a.w[i] = greedy ? v : __fmul_rn(v, P.inv_temp);
    }
    if (P.rep > 1.0f) {
        if (tid == 0) sm.n_owner = 0;
        __syncthreads();
        const int hl = s->hist_len;
        for (int h = tid; h < hl; h += ST) {
            const int t = a.hist[h];
            if (t >= 0 && t < V && atomicAdd(&a.cnt[t], 1) == 0) sm.u.owners[atomicAdd(&sm.n_owner, 1)] = t;
        }
        __syncthreads();
        for (int j = tid; j < sm.n_owner; j += ST) {
            const int t = sm.u.owners[j];
            const int c = atomicExch(&a.cnt[t], 0);
            float x = a.logits[t];
            for (int q = 0; q < c; ++q) x = x > 0.0f ? __fdiv_rn(x, P.rep) : __fmul_rn(x, P.rep);
            a.w[t] = greedy ? x : __fmul_rn(x, P.inv_temp);
        }
    }
    __syncthreads();
    if (greedy) {  // picchio.c:1555-1562
        emit(a, block_argmax(a.w, V, sm), true);
        return;
    }

    // top-k (picchio.c:1571-1581): values below the k-th largest -> -1e30
    const bool topk = P.top_k > 0 && P.top_k < V;
    const float th = topk ? kth_largest(a.w, V, P.top_k, sm) : 0.0f;
    // softmax (picchio.c:1584-1591)
    float mx = -1e30f;
    for (int i = tid; i < V; i += ST) {
        float v = a.w[i];
        if (topk && v < th) {
            v = -1e30f;
            a.w[i] = v;
        }
        mx = v > mx ? v : mx;
    }
    mx = block_max(mx, sm);
    int n_nz = 0;  // exponentials, compacted in index order
    for (int base = 0; base < V; base += ST * 4) {
        float e[4];
        int c = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int i = base + tid * 4 + k;
            e[k] = 0.0f;
            if (i < V) {
                const float d = __fsub_rn(a.w[i], mx);
                e[k] = d < -104.0f ? 0.0f : __double2float_rn(exp((double)d));  // below -104: under half of 2^-149
            }
            c += e[k] != 0.0f;
        }
        int total;
        int o = n_nz + block_excl_scan(c, &total, sm);
#pragma unroll
        for (int k = 0; k < 4; ++k)
            if (e[k] != 0.0f) {
                a.nz_val[o] = e[k];
                a.nz_idx[o] = base + tid * 4 + k;
                ++o;
            }
        n_nz += total;
    }
    __syncthreads();
    const float sum = seq_sum(a.nz_val, n_nz, sm);
    for (int j = tid; j < n_nz; j += ST) a.nz_val[j] = __fdiv_rn(a.nz_val[j], sum);
    __syncthreads();

    // top-p (picchio.c:1594-1627)
    if (P.top_p < 1.0f && P.top_p > 0.0f) {
        int c = 0;
        for (int j = tid; j < n_nz; j += ST) c += a.nz_val[j] > 1e-10f;
        const int n_c = block_sum_i(c, sm);
        if (n_c > 1) {
            if (n_c > SAMPLE_SORT_CAP) {
                if (!a.big) {  // the host did not provide the large sort
                    if (tid == 0) {
                        s->status = 1;
                        if (a.err) atomicExch(a.err, SAMPLE_ERR_CANDIDATES);
                    }
                    emit(a, 0, false);
                    return;
                }
                for (int j = tid; j < V; j += ST) {
                    const float v = j < n_nz ? a.nz_val[j] : 0.0f;
                    a.ck[j] = v > 1e-10f ? v : -1.0f;
                    a.cv[j] = j;
                }
                if (tid == 0) {
                    s->stage = 1;
                    s->n_nz = n_nz;
                    s->n_cand = n_c;
                }
                return;
            }
            // candidates in index order, then a bitonic sort: descending
            // probability, ties by id
            int P2 = 2;
            while (P2 < n_c) P2 <<= 1;
            int nfill = 0;
            for (int base = 0; base < n_nz; base += ST) {
                const int j = base + tid;
                const bool f = j < n_nz && a.nz_val[j] > 1e-10f;
                int total;
                const int o = nfill + block_excl_scan(f ? 1 : 0, &total, sm);
                if (f) {
                    sm.u.cand.key[o] = a.nz_val[j];
                    sm.u.cand.pos[o] = j;
                }
                nfill += total;
            }
            for (int j = n_c + tid; j < P2; j += ST) {
                sm.u.cand.key[j] = -1.0f;
                sm.u.cand.pos[j] = INT_MAX;
            }
            __syncthreads();
            for (int size = 2; size <= P2; size <<= 1) {
                for (int stride = size >> 1; stride > 0; stride >>= 1) {
                    for (int t = tid; t < P2 / 2; t += ST) {
                        const int lo = 2 * t - (t & (stride - 1)), hi = lo + stride;
                        const float kl = sm.u.cand.key[lo], kh = sm.u.cand.key[hi];
                        const int pl = sm.u.cand.pos[lo], ph = sm.u.cand.pos[hi];
                        const bool hi_first = kh > kl || (kh == kl && ph < pl);
                        const bool lo_first = kl > kh || (kl == kh && pl < ph);
                        if ((lo & size) == 0 ? hi_first : lo_first) {
                            sm.u.cand.key[lo] = kh;
                            sm.u.cand.key[hi] = kl;
                            sm.u.cand.pos[lo] = ph;
                            sm.u.cand.pos[hi] = pl;
                        }
                    }
                    __syncthreads();
                }
            }
            int cut = n_c;
            if (tid == 0) {
                float cum = 0.0f;
                for (int i = 0; i < n_c; ++i) {
                    cum = __fadd_rn(cum, sm.u.cand.key[i]);
                    if (cum >= P.top_p) { cut = i + 1; break; }
                }
                sm.bi[2] = cut;
            }
            __syncthreads();
            cut = sm.bi[2];
            apply_cut(a, n_nz, sm.u.cand.pos, cut, n_c, sm);
        }
    }
    draw(a, n_nz, sm);
}

// Continuation after the large sort of the top-p candidates (sk / sv: keys
// descending, equal keys in position order).
__global__ void __launch_bounds__(ST, 1) sample_tail_kernel(const SampleArgs a) {
    __shared__ SampleSmem sm;
    pdl_wait();
    pdl_trigger();
    SampleState *s = a.s;
    if (s->stage != 1) return;
    const int n_nz = s->n_nz, n_c = s->n_cand;
    const int cut = seq_cut(a.sk, n_c, s->p.top_p, sm);
    apply_cut(a, n_nz, a.sv, cut, n_c, sm);
    draw(a, n_nz, sm);
    if (threadIdx.x == 0) s->stage = 0;
}

}  // namespace

cudaError_t sampler_init(Sampler &s, int V) {
    if (s.state) return cudaSuccess;
    s.V = V;
    cudaError_t e = cudaMalloc(&s.state, sizeof(SampleState));
    if (e == cudaSuccess) e = cudaMemset(s.state, 0, sizeof(SampleState));
    if (e == cudaSuccess) e = cudaMalloc(&s.hist, SAMPLE_HIST_CAP * sizeof(int));
    if (e == cudaSuccess) e = cudaMalloc(&s.cnt, (size_t)V * sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(s.cnt, 0, (size_t)V * sizeof(int));
    if (e == cudaSuccess) e = cudaMalloc(&s.w, (size_t)V * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&s.nz_val, (size_t)V * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&s.nz_idx, (size_t)V * sizeof(int));
    if (e == cudaSuccess) e = cudaMalloc(&s.ck, (size_t)V * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&s.sk, (size_t)V * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&s.cv, (size_t)V * sizeof(int));
    if (e == cudaSuccess) e = cudaMalloc(&s.sv, (size_t)V * sizeof(int));
    if (e == cudaSuccess)
        e = cub::DeviceRadixSort::SortPairsDescending(nullptr, s.tmp_bytes, s.ck, s.sk, s.cv, s.sv, V);
    if (e == cudaSuccess) e = cudaMalloc(&s.tmp, s.tmp_bytes);
    // the memsets above run on the legacy default stream, which a
    // context's non-blocking stream does not wait for
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    return e;
}

void sampler_free(Sampler &s) {
    void *p[] = {s.state, s.hist, s.cnt, s.w, s.nz_val, s.nz_idx, s.ck, s.sk, s.cv, s.sv, s.tmp};
    for (void *q : p)
        if (q) cudaFree(q);
    s = Sampler{};
}

cudaError_t sampler_launch(const Sampler &s, const float *logits, int *ids, int *ids2, int *err, cudaStream_t st,
                           int &launches) {
    SampleArgs a{};
    a.err = err;
    a.logits = logits;
    a.V = s.V;
    a.big = s.big ? 1 : 0;
    a.s = s.state;
    a.hist = s.hist;
    a.cnt = s.cnt;
    a.w = s.w;
    a.nz_val = s.nz_val;
    a.nz_idx = s.nz_idx;
    a.ck = s.ck;
    a.cv = s.cv;
    a.sk = s.sk;
    a.sv = s.sv;
    a.ids = ids;
    a.ids2 = ids2;
    cudaError_t e = launch_k(sample_kernel, dim3(1), dim3(ST), 0, st, a);
    ++launches;
    if (e != cudaSuccess || !s.big) return e;
    size_t bytes = s.tmp_bytes;
    e = cub::DeviceRadixSort::SortPairsDescending(s.tmp, bytes, s.ck, s.sk, s.cv, s.sv, s.V, 0, 32, st);
    if (e != cudaSuccess) return e;
    e = launch_k(sample_tail_kernel, dim3(1), dim3(ST), 0, st, a);
    ++launches;
    return e;
}

}  // namespace pc
