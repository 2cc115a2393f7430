// Token selection from float32 logits, one block per row.
//   temperature == 0          the largest logit; among equal ones the lowest token id.
//   temperature > 0           softmax(logits / temperature) in float32 and an inverse-CDF draw
//                             with u in [0, 1) taken from (seed, counter) alone, so that a
//                             request's stream does not depend on its place in the batch.
//   top_k in 1..SAMPLE_MAX_K  only the k largest logits take part (lowest id first among equal
//                             ones); they are walked from the largest down. The candidates are found in two
//                             kernels: the vocabulary is cut into 32 slices, a block per slice and row selects
//                             the slice's k largest by a radix select over an order-preserving 32-bit key (four
//                             rounds of 256-bin histograms in shared memory, no sorting), and a block per row
//                             selects the k largest of those, ranks them and draws. (A row whose vocabulary
//                             does not fit the slices' shared memory is served by the row's own block, one
//                             block-wide selection per candidate.)
//   top_p < 1                 of those, the low tail whose cumulative probability is <= 1 - top_p
//                             is left out; the largest always stays.
//   top_k > SAMPLE_MAX_K, or top_p < 1 without top_k: the cuts are found as thresholds on the logit's
//                             value, by a radix descent over the 32 bits of an order-preserving key
//                             (rounds of 12, 12 and 8 bits with a histogram in shared memory; no sorting):
//                             first the value of the k-th largest logit, everything below it is out;
//                             then the largest value t such that the logits below t (of those still in)
//                             hold at most 1 - top_p of the probability (weighed in fixed point, all of it
//                             about 2^31, so that the sums do not depend on the order of the additions), and
//                             everything below t is out. Logits equal to a threshold all stay. The draw
//                             walks the vocabulary in id order.
#include "common.cuh"

#define SAMPLE_THREADS 1024
#define SAMPLE_MAX_K 64

__host__ __device__ __forceinline__ float uniform_from(uint64_t seed, uint64_t counter) {
    uint64_t x = seed ^ (counter + 0x9E3779B97F4A7C15ull);
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    x = x ^ (x >> 31);
    return (float)(x >> 40) * (1.0f / 16777216.0f);
}

// float -> unsigned key with the same order (larger float, larger key)
__device__ __forceinline__ uint32_t ordered_key(float f) {
    const uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

struct Best {
    float value;
    int index;
};
__device__ __forceinline__ Best better(Best a, Best b) {   // larger value, then lower index
    if (b.value > a.value || (b.value == a.value && b.index < a.index)) return b;
    return a;
}
__device__ __forceinline__ Best block_best(Best v, Best* scratch) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        Best other;
        other.value = __shfl_xor_sync(0xffffffffu, v.value, o);
        other.index = __shfl_xor_sync(0xffffffffu, v.index, o);
        v = better(v, other);
    }
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    Best r = (lane < nwarps) ? scratch[lane] : Best{-INFINITY, 0x7fffffff};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        Best other;
        other.value = __shfl_xor_sync(0xffffffffu, r.value, o);
        other.index = __shfl_xor_sync(0xffffffffu, r.index, o);
        r = better(r, other);
    }
    return r;
}

// ---- thresholds on the value by radix descent (the general path of sample_kernel)
#define RADIX_BINS 4096            // twelve bits a round; the key's 32 bits in rounds of 12, 12 and 8

// Block-wide exclusive prefix sums of one 64-bit value per thread, in thread order; `total`: the sum of all.
__device__ unsigned long long block_scan_u64(unsigned long long v, unsigned long long* scratch /* 33 */, unsigned long long* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    unsigned long long inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long up = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += up;
    }
    __syncthreads();
    if (lane == 31) scratch[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        const unsigned long long w = lane < nwarps ? scratch[lane] : 0ull;
        unsigned long long winc = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned long long up = __shfl_up_sync(0xffffffffu, winc, o);
            if (lane >= o) winc += up;
        }
        scratch[lane] = winc - w;
        if (lane == 31) scratch[32] = winc;
    }
    __syncthreads();
    *total = scratch[32];
    return scratch[warp] + inc - v;
}

// The weight a logit adds to a histogram: 1 when logits are counted; when probability mass is weighed, its
// probability in fixed point, scaled so that all logits together weigh about 2^31 (`mass_scale` = 2^31 / sum of
// exp): integers, so that sums do not depend on the order of the additions, and 32 bits, so that shared-memory
// atomics take them natively.
__device__ __forceinline__ uint32_t radix_weight(float v, float top_value, float inv_temp, float mass_scale) {
    return mass_scale > 0.f ? (uint32_t)(expf((v - top_value) * inv_temp) * mass_scale) : 1u;
}

// A descent over the bits of the order-preserving key, twelve (then eight) at a time, with a histogram of
// RADIX_BINS 64-bit counters in shared memory per round. Logits with a key below `cut` take no part.
//   mass false: the key of the `want`-th largest logit (1 <= want <= logits taking part).
//   mass true:  the largest key t such that the logits with keys below t weigh at most `want` together.
// Every thread of the block calls it and gets the result.
__device__ uint32_t block_radix_descent(const float* __restrict__ l, int vocab, uint32_t cut, float top_value, float inv_temp,
                                        float mass_scale, unsigned long long want, uint32_t* hist,
                                        unsigned long long* scratch /* 33 */, uint32_t* state /* 2 */,
                                        unsigned long long* state64 /* 1 */) {
    const int tid = threadIdx.x, threads = blockDim.x;
    const bool mass = mass_scale > 0.f;
    if (tid == 0) { state[0] = 0u; state[1] = 0u; state64[0] = want; }
    __syncthreads();
    const int shifts[3] = {20, 8, 0}, widths[3] = {12, 12, 8};
    for (int round = 0; round < 3; ++round) {
        const int shift = shifts[round], bins = 1 << widths[round];
        for (int b = tid; b < bins; b += threads) hist[b] = 0u;
        __syncthreads();
        const uint32_t prefix = state[0], mask = state[1];
        const unsigned long long left = state64[0];          // still to find (count) / still allowed below (mass)
        for (int base = 0; base < vocab; base += 4 * threads) {      // four loads in flight at a time
            float v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = base + u * threads + tid;
                v[u] = i < vocab ? l[i] : 0.f;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = base + u * threads + tid;
                const uint32_t key = ordered_key(v[u]);
                if (i < vocab && key >= cut && (key & mask) == prefix)
                    atomicAdd(&hist[(key >> shift) & (uint32_t)(bins - 1)], radix_weight(v[u], top_value, inv_temp, mass_scale));
            }
        }
        __syncthreads();
        // thread t owns `per` consecutive bins, taken from the top when counting and from the bottom when weighing
        const int per = (bins + threads - 1) / threads;
        unsigned long long mine = 0ull;
        for (int j = 0; j < per; ++j) {
            const int pos = tid * per + j;
            if (pos < bins) mine += hist[mass ? pos : bins - 1 - pos];
        }
        unsigned long long total;
        unsigned long long before = block_scan_u64(mine, scratch, &total);
        // counting: the bin at which the count from the top reaches `left`; weighing: the last bin that can be
        // reached with at most `left` below it
        for (int j = 0; j < per; ++j) {
            const int pos = tid * per + j;
            if (pos >= bins) break;
            const int bin = mass ? pos : bins - 1 - pos;
            const unsigned long long h = hist[bin];
            bool chosen;
            if (mass) {
                const bool last = pos == bins - 1;
                chosen = before <= left && (last || before + h > left);     // the next bin would have more than `left` below it
            } else {
                chosen = before < left && before + h >= left;
            }
            if (chosen) {
                state[0] = prefix | ((uint32_t)bin << shift);
                state[1] = mask | ((uint32_t)(bins - 1) << shift);
                state64[0] = left - before;
            }
            before += h;
        }
        __syncthreads();
    }
    return state[0];
}

__global__ void __launch_bounds__(SAMPLE_THREADS)
sample_kernel(const float* __restrict__ logits, int ld, int vocab, const float* __restrict__ temperature,
              const int* __restrict__ top_k, const float* __restrict__ top_p, const long long* __restrict__ seeds,
              const int* __restrict__ counters, int* __restrict__ out, int skip_sliced) {
    __shared__ Best best_scratch[32];
    __shared__ float sum_scratch[32];
    __shared__ float chunk_sum[SAMPLE_THREADS];
    __shared__ float cand_value[SAMPLE_MAX_K];
    __shared__ int cand_index[SAMPLE_MAX_K];
    __shared__ int result;
    extern __shared__ uint32_t radix_hist[];                 // RADIX_BINS counters of the general path
    __shared__ unsigned long long scan_scratch[33], radix_state64[1];
    __shared__ uint32_t radix_state[2];
    pdl_wait();
    pdl_launch_dependents();
    const int row = blockIdx.x;
    const float* l = logits + (size_t)row * ld;
    const int tid = threadIdx.x;
    if (skip_sliced && temperature && temperature[row] > 0.f && top_k && top_k[row] >= 1 && top_k[row] <= SAMPLE_MAX_K)
        return;                                   // the sliced top-k kernels serve this row

    Best mine{-INFINITY, 0x7fffffff};
    for (int base = tid; base < vocab; base += 4 * SAMPLE_THREADS) {       // four loads in flight at a time
        float v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) v[u] = base + u * SAMPLE_THREADS < vocab ? l[base + u * SAMPLE_THREADS] : -INFINITY;
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (base + u * SAMPLE_THREADS < vocab) mine = better(mine, Best{v[u], base + u * SAMPLE_THREADS});
    }
    const Best top = block_best(mine, best_scratch);
    const float temp = temperature ? temperature[row] : 0.f;
    if (!(temp > 0.f)) {
        if (tid == 0) out[row] = top.index;
        return;
    }
    const float inv_temp = 1.f / temp;
    const float u = uniform_from((uint64_t)seeds[row], (uint64_t)(uint32_t)counters[row]);
    int k = top_k ? top_k[row] : 0;
    if (k > vocab) k = vocab;

    const float p_limit = top_p ? top_p[row] : 1.f;
    if (k <= 0 || k > SAMPLE_MAX_K) {
        // ---- the cuts as thresholds on the value (see the head of this file); cut = 0 keeps everything
        uint32_t cut = 0;
        const uint32_t top_key = ordered_key(top.value);
        if (k > SAMPLE_MAX_K && k < vocab)      // the key of the k-th largest logit: everything below it is out
            cut = block_radix_descent(l, vocab, 0u, top.value, inv_temp, 0.f, (unsigned long long)k, radix_hist, scan_scratch,
                                      radix_state, radix_state64);
        if (p_limit < 1.f) {
            // what is still in weighs about 2^31 in fixed point; then the largest key t with at most (1 - top_p) of
            // that weight below t
            float kept = 0.f;
            for (int base = tid; base < vocab; base += 4 * SAMPLE_THREADS) {
                float v[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) v[u] = base + u * SAMPLE_THREADS < vocab ? l[base + u * SAMPLE_THREADS] : -INFINITY;
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    if (ordered_key(v[u]) >= cut) kept += expf((v[u] - top.value) * inv_temp);      // -inf weighs nothing
            }
            kept = block_sum(kept, sum_scratch);
            const float mass_scale = 2147483648.f / kept;
            unsigned long long weight = 0ull;
            for (int base = tid; base < vocab; base += 4 * SAMPLE_THREADS) {
                float v[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) v[u] = base + u * SAMPLE_THREADS < vocab ? l[base + u * SAMPLE_THREADS] : -INFINITY;
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    if (base + u * SAMPLE_THREADS < vocab && ordered_key(v[u]) >= cut)
                        weight += radix_weight(v[u], top.value, inv_temp, mass_scale);
            }
            unsigned long long total;
            block_scan_u64(weight, scan_scratch, &total);
            const unsigned long long limit = (unsigned long long)((double)total * (1.0 - (double)p_limit));
            const uint32_t t = block_radix_descent(l, vocab, cut, top.value, inv_temp, mass_scale, limit, radix_hist, scan_scratch,
                                                   radix_state, radix_state64);
            cut = t < top_key ? t : top_key;              // the largest logit always stays
        }
        // ---- the draw: thread `tid` owns the contiguous ids [tid * chunk, (tid + 1) * chunk)
        const int chunk = (vocab + SAMPLE_THREADS - 1) / SAMPLE_THREADS;
        const int begin = tid * chunk, end = min(begin + chunk, vocab);
        float s = 0.f;
        for (int i = begin; i < end; ++i)
            if (ordered_key(l[i]) >= cut) s += expf((l[i] - top.value) * inv_temp);
        __syncthreads();
        chunk_sum[tid] = s;
        if (tid == 0) result = -1;
        __syncthreads();
        if (tid == 0) {   // serial prefix over 1024 chunk sums: same numbers, same order, on every run
            float running = 0.f;
            for (int c = 0; c < SAMPLE_THREADS; ++c) {
                const float before = running;
                running += chunk_sum[c];
                chunk_sum[c] = before;
            }
            sum_scratch[0] = running;
        }
        __syncthreads();
        const float total = sum_scratch[0];
        const float target = u * total;
        const float before = chunk_sum[tid];
        const float after = (tid + 1 < SAMPLE_THREADS) ? chunk_sum[tid + 1] : total;
        if (begin < end && target >= before && (target < after || end == vocab)) {
            float running = before;
            int pick = -1, last_positive = -1;
            for (int i = begin; i < end; ++i) {
                if (ordered_key(l[i]) < cut) continue;
                const float p = expf((l[i] - top.value) * inv_temp);
                running += p;
                if (p > 0.f) last_positive = i;
                if (running > target) { pick = i; break; }
            }
            if (pick < 0) pick = last_positive;
            if (pick >= 0) atomicMax(&result, pick);
        }
        __syncthreads();
        if (tid == 0) out[row] = result >= 0 ? result : top.index;
        return;
    }

    // the k largest, one block-wide selection per candidate
    Best previous = top;
    if (tid == 0) { cand_value[0] = top.value; cand_index[0] = top.index; }
    for (int c = 1; c < k; ++c) {
        Best m{-INFINITY, 0x7fffffff};
        for (int i = tid; i < vocab; i += SAMPLE_THREADS) {
            const float v = l[i];
            const bool after_previous = v < previous.value || (v == previous.value && i > previous.index);
            if (after_previous) m = better(m, Best{v, i});
        }
        previous = block_best(m, best_scratch);
        if (tid == 0) { cand_value[c] = previous.value; cand_index[c] = previous.index; }
    }
    __syncthreads();
    if (tid == 0) {
        float prob[SAMPLE_MAX_K];
        float total = 0.f;
        for (int c = 0; c < k; ++c) { prob[c] = expf((cand_value[c] - top.value) * inv_temp); total += prob[c]; }
        int keep = k;
        if (p_limit < 1.f) {
            float tail = 0.f;
            for (int c = k - 1; c >= 1; --c) {
                tail += prob[c] / total;
                if (tail <= 1.f - p_limit) keep = c; else break;
            }
        }
        float kept_total = 0.f;
        for (int c = 0; c < keep; ++c) kept_total += prob[c];
        const float target = u * kept_total;
        float running = 0.f;
        int pick = cand_index[keep - 1];
        for (int c = 0; c < keep; ++c) {
            running += prob[c];
            if (running > target) { pick = cand_index[c]; break; }
        }
        out[row] = pick;
    }
}

// ---- top_k up to SAMPLE_MAX_K: the slices' candidates, then the row's
#define TOPK_SLICES 32
#define TOPK_THREADS 256
#define TOPK_MAX_SLICE 8192          // logits of a slice held in shared memory as keys

// The key of the k-th largest of keys[0..n) (1 <= k <= n), by four rounds of 256-bin histograms over the bits of
// the key from the top; *ties: how many of the keys equal to it belong to the k largest. hist: 256 counters,
// state: 3 words, both in shared memory. Every thread of the block calls it and gets the result.
__device__ uint32_t block_kth_largest_key(const uint32_t* keys, int n, int k, uint32_t* hist, uint32_t* state, int* ties) {
    const int tid = threadIdx.x, threads = blockDim.x;
    if (tid == 0) { state[0] = 0u; state[1] = 0u; state[2] = (uint32_t)k; }      // prefix, mask, still to find
    __syncthreads();
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int b = tid; b < 256; b += threads) hist[b] = 0u;
        __syncthreads();
        const uint32_t prefix = state[0], mask = state[1], want = state[2];     // read before anybody writes them again
        for (int i = tid; i < n; i += threads) {
            const uint32_t key = keys[i];
            if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (tid < 32) {
            // lane l owns bins 8l .. 8l + 7; the bin sought is the highest one at which the count from the top
            // reaches what is still to find
            uint32_t local = 0;
#pragma unroll
            for (int b = 0; b < 8; ++b) local += hist[tid * 8 + b];
            uint32_t above = 0;                               // keys in the bins of higher lanes
            for (int src = 0; src < 32; ++src) {              // every lane takes part in every shuffle
                const uint32_t theirs = __shfl_sync(0xffffffffu, local, src);
                if (src > tid) above += theirs;
            }
            const bool here = above < want && above + local >= want;
            if (here) {
                uint32_t cum = above;
                int bin = tid * 8 + 7;
                for (; bin > tid * 8; --bin) {
                    if (cum + hist[bin] >= want) break;
                    cum += hist[bin];
                }
                state[0] = prefix | ((uint32_t)bin << shift);
                state[1] = mask | (255u << shift);
                state[2] = want - cum;
            }
        }
        __syncthreads();
    }
    *ties = (int)state[2];
    return state[0];
}

// Exclusive prefix sums over the block of two small counts per thread (a, b <= 65535 in total each), in thread order.
__device__ void block_scan_pair(int a, int b, int* a_before, int* b_before, uint32_t* scratch /* 33 words */) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    uint32_t v = (uint32_t)a | ((uint32_t)b << 16), inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t up = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += up;
    }
    __syncthreads();
    if (lane == 31) scratch[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        uint32_t w = lane < nwarps ? scratch[lane] : 0u, winc = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t up = __shfl_up_sync(0xffffffffu, winc, o);
            if (lane >= o) winc += up;
        }
        scratch[lane] = winc - w;                             // exclusive over the warps
    }
    __syncthreads();
    const uint32_t before = scratch[warp] + inc - v;
    *a_before = (int)(before & 0xffffu);
    *b_before = (int)(before >> 16);
}

struct Cand {
    float value;
    int index;
};

// Of keys[0..n) with ids id0 + i: the k largest (k <= n), among equal ones those that come first, written to
// out[0..k) (the larger ones in the order they come, then the ties in the order they come).
__device__ void block_select_top(const uint32_t* keys, const float* values, const int* ids, int id0, int n, int k, Cand* out,
                                 uint32_t* hist, uint32_t* state, uint32_t* scratch) {
    int ties = 0;
    const uint32_t t = block_kth_largest_key(keys, n, k, hist, state, &ties);
    const int larger = k - ties;
    const int per = (n + blockDim.x - 1) / blockDim.x;
    const int begin = min(n, (int)threadIdx.x * per), end = min(n, begin + per);
    int g = 0, e = 0;
    for (int i = begin; i < end; ++i) {
        g += keys[i] > t ? 1 : 0;
        e += keys[i] == t ? 1 : 0;
    }
    int g_before, e_before;
    block_scan_pair(g, e, &g_before, &e_before, scratch);
    for (int i = begin; i < end; ++i) {
        const uint32_t key = keys[i];
        if (key > t) {
            out[g_before++] = Cand{values[i], ids ? ids[i] : id0 + i};
        } else if (key == t) {
            if (e_before < ties) out[larger + e_before] = Cand{values[i], ids ? ids[i] : id0 + i};
            ++e_before;
        }
    }
}

// One block per (slice, row): the slice's min(k, slice length) largest logits -> cand[row][slice][..], their number
// -> count[row][slice]. Rows that are greedy, or whose top_k lies outside 1..SAMPLE_MAX_K, are left alone.
__global__ void __launch_bounds__(TOPK_THREADS)
topk_slices_kernel(const float* __restrict__ logits, int ld, int vocab, const float* __restrict__ temperature,
                   const int* __restrict__ top_k, Cand* __restrict__ cand, int* __restrict__ count) {
    extern __shared__ uint32_t slice_keys[];              // [per] keys, then [per] values
    __shared__ uint32_t hist[256], state[3], scratch[33];
    __shared__ Cand picked[SAMPLE_MAX_K];
    pdl_wait();
    pdl_launch_dependents();
    const int slice = blockIdx.x, row = blockIdx.y, tid = threadIdx.x;
    const int k_row = top_k[row];
    if (!(temperature[row] > 0.f) || k_row < 1 || k_row > SAMPLE_MAX_K) return;
    const int per = ((vocab + TOPK_SLICES - 1) / TOPK_SLICES + 3) & ~3;
    const int id0 = slice * per, n = max(0, min(vocab, id0 + per) - id0);
    float* slice_values = reinterpret_cast<float*>(slice_keys + per);
    const float* l = logits + (size_t)row * ld + id0;
    for (int i = tid; i < n; i += TOPK_THREADS) {
        const float v = l[i];
        slice_values[i] = v;
        slice_keys[i] = ordered_key(v);
    }
    __syncthreads();
    const int k = min(k_row, n);
    if (k > 0) block_select_top(slice_keys, slice_values, nullptr, id0, n, k, picked, hist, state, scratch);
    __syncthreads();
    Cand* dst = cand + ((size_t)row * TOPK_SLICES + slice) * SAMPLE_MAX_K;
    for (int i = tid; i < k; i += TOPK_THREADS) dst[i] = picked[i];
    if (tid == 0) count[row * TOPK_SLICES + slice] = k;
}

// One block per row: the k largest of the slices' candidates (taken slice by slice, so that equal logits keep
// the order of their ids), ranked from the largest down; then probabilities, the top_p cut and the draw.
__global__ void __launch_bounds__(TOPK_THREADS)
topk_draw_kernel(const Cand* __restrict__ cand, const int* __restrict__ count, int vocab,
                 const float* __restrict__ temperature, const int* __restrict__ top_k, const float* __restrict__ top_p,
                 const long long* __restrict__ seeds, const int* __restrict__ counters, int* __restrict__ out) {
    __shared__ uint32_t keys[TOPK_SLICES * SAMPLE_MAX_K];
    __shared__ float values[TOPK_SLICES * SAMPLE_MAX_K];
    __shared__ int ids[TOPK_SLICES * SAMPLE_MAX_K];
    __shared__ int offset[TOPK_SLICES + 1];
    __shared__ uint32_t hist[256], state[3], scratch[33];
    __shared__ Cand picked[SAMPLE_MAX_K], ranked[SAMPLE_MAX_K];
    pdl_wait();
    pdl_launch_dependents();
    const int row = blockIdx.x, tid = threadIdx.x;
    const int k_row = top_k[row];
    const float temp = temperature[row];
    if (!(temp > 0.f) || k_row < 1 || k_row > SAMPLE_MAX_K) return;
    if (tid == 0) {
        int total = 0;
        for (int s = 0; s < TOPK_SLICES; ++s) { offset[s] = total; total += count[row * TOPK_SLICES + s]; }
        offset[TOPK_SLICES] = total;
    }
    __syncthreads();
    const int n = offset[TOPK_SLICES];
    for (int i = tid; i < TOPK_SLICES * SAMPLE_MAX_K; i += TOPK_THREADS) {
        const int s = i / SAMPLE_MAX_K, j = i % SAMPLE_MAX_K;
        if (j < offset[s + 1] - offset[s]) {
            const Cand c = cand[((size_t)row * TOPK_SLICES + s) * SAMPLE_MAX_K + j];
            values[offset[s] + j] = c.value;
            ids[offset[s] + j] = c.index;
            keys[offset[s] + j] = ordered_key(c.value);
        }
    }
    __syncthreads();
    const int k = min(min(k_row, vocab), n);
    if (k <= 0) {
        if (tid == 0) out[row] = 0;
        return;
    }
    block_select_top(keys, values, ids, 0, n, k, picked, hist, state, scratch);
    __syncthreads();
    // rank: how many candidates are better (a larger logit, or the same logit and a lower id)
    if (tid < k) {
        const Cand me = picked[tid];
        int rank = 0;
        for (int j = 0; j < k; ++j) {
            const Cand other = picked[j];
            rank += (other.value > me.value || (other.value == me.value && other.index < me.index)) ? 1 : 0;
        }
        ranked[rank] = me;
    }
    __syncthreads();
    if (tid == 0) {
        const float inv_temp = 1.f / temp;
        const float u = uniform_from((uint64_t)seeds[row], (uint64_t)(uint32_t)counters[row]);
        const float p_limit = top_p ? top_p[row] : 1.f;
        const float top_value = ranked[0].value;
        float prob[SAMPLE_MAX_K];
        float total = 0.f;
        for (int c = 0; c < k; ++c) { prob[c] = expf((ranked[c].value - top_value) * inv_temp); total += prob[c]; }
        int keep = k;
        if (p_limit < 1.f) {
            float tail = 0.f;
            for (int c = k - 1; c >= 1; --c) {
                tail += prob[c] / total;
                if (tail <= 1.f - p_limit) keep = c; else break;
            }
        }
        float kept_total = 0.f;
        for (int c = 0; c < keep; ++c) kept_total += prob[c];
        const float target = u * kept_total;
        float running = 0.f;
        int pick = ranked[keep - 1].index;
        for (int c = 0; c < keep; ++c) {
            running += prob[c];
            if (running > target) { pick = ranked[c].index; break; }
        }
        out[row] = pick;
    }
}

// ---- the largest logit of every row, the vocabulary cut into ARGMAX_PARTS slices of one block each
// (one block per row, as above, is bound by the latency of a single block's loads at a vocabulary of 128 K)
#define ARGMAX_PARTS 32
#define ARGMAX_THREADS 256

__global__ void __launch_bounds__(ARGMAX_THREADS)
argmax_partial_kernel(const float* __restrict__ logits, int ld, int vocab, Best* __restrict__ partial) {
    __shared__ Best scratch[32];
    pdl_wait();
    pdl_launch_dependents();
    const int row = blockIdx.y, part = blockIdx.x;
    const float* l = logits + (size_t)row * ld;
    const int per = ((vocab + ARGMAX_PARTS - 1) / ARGMAX_PARTS + 3) & ~3;       // a multiple of four ids
    const int begin = part * per, end = min(begin + per, vocab);
    Best mine{-INFINITY, 0x7fffffff};
    if ((ld & 3) == 0 && (reinterpret_cast<uintptr_t>(logits) & 15) == 0) {
        const int end4 = begin + ((end - begin) > 0 ? ((end - begin) & ~3) : 0);
        for (int i = begin + 4 * threadIdx.x; i < end4; i += 4 * ARGMAX_THREADS) {
            const float4 v = *reinterpret_cast<const float4*>(l + i);
            mine = better(mine, Best{v.x, i});
            mine = better(mine, Best{v.y, i + 1});
            mine = better(mine, Best{v.z, i + 2});
            mine = better(mine, Best{v.w, i + 3});
        }
        for (int i = end4 + threadIdx.x; i < end; i += ARGMAX_THREADS) mine = better(mine, Best{l[i], i});
    } else {
        for (int i = begin + threadIdx.x; i < end; i += ARGMAX_THREADS) mine = better(mine, Best{l[i], i});
    }
    const Best top = block_best(mine, scratch);
    if (threadIdx.x == 0) partial[row * ARGMAX_PARTS + part] = top;
}

// one warp per row
__global__ void argmax_final_kernel(const Best* __restrict__ partial, int rows, int* __restrict__ out) {
    pdl_wait();
    pdl_launch_dependents();
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    Best v = lane < ARGMAX_PARTS ? partial[row * ARGMAX_PARTS + lane] : Best{-INFINITY, 0x7fffffff};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        Best other;
        other.value = __shfl_xor_sync(0xffffffffu, v.value, o);
        other.index = __shfl_xor_sync(0xffffffffu, v.index, o);
        v = better(v, other);
    }
    if (lane == 0) out[row] = v.index;
}

TTB_EXPORT int ttb_argmax_scratch_bytes(int rows) { return rows * ARGMAX_PARTS * (int)sizeof(Best); }

// out[row] = the id of the row's largest logit (the lowest id among equal ones); scratch: ttb_argmax_scratch_bytes(rows).
TTB_EXPORT int ttb_argmax(const float* logits, int ld, int rows, int vocab, void* scratch, int* out, cudaStream_t stream) {
    if (rows == 0) return TTB_OK;
    if (!logits || !out || !scratch || vocab < 1) return TTB_ERR_ARGUMENT;
    if (rows > 65535) return TTB_ERR_UNSUPPORTED;
    static_assert(ARGMAX_PARTS <= 32, "the final kernel reads one partial result per lane");
    ttb_launch(argmax_partial_kernel, dim3(ARGMAX_PARTS, rows), dim3(ARGMAX_THREADS), 0, stream, logits, ld, vocab,
               (Best*)scratch);
    int status = ttb_launch_status();
    if (status != TTB_OK) return status;
    ttb_launch(argmax_final_kernel, dim3((rows + 3) / 4), dim3(128), 0, stream, (const Best*)scratch, rows, out);
    return ttb_launch_status();
}

// Scratch memory that ttb_sample wants for `rows` rows when top_k is given (the slices' candidates and their counts).
TTB_EXPORT int ttb_sample_scratch_bytes(int rows) {
    return rows * TOPK_SLICES * (SAMPLE_MAX_K * (int)sizeof(Cand) + (int)sizeof(int));
}

// scratch: ttb_sample_scratch_bytes(rows) bytes, or null (then every row is served by its own block).
TTB_EXPORT int ttb_sample(const float* logits, int ld, int rows, int vocab, const float* temperature,
                          const int* top_k, const float* top_p, const long long* seeds, const int* counters,
                          int* out, void* scratch, cudaStream_t stream) {
    if (rows == 0) return TTB_OK;
    if (!logits || !out || vocab < 1) return TTB_ERR_ARGUMENT;
    if (temperature && (!seeds || !counters)) return TTB_ERR_ARGUMENT;
    const int per = ((vocab + TOPK_SLICES - 1) / TOPK_SLICES + 3) & ~3;
    const bool sliced = scratch && temperature && top_k && per <= TOPK_MAX_SLICE && rows <= 65535;
    if (sliced) {
        Cand* cand = static_cast<Cand*>(scratch);
        int* count = reinterpret_cast<int*>(cand + (size_t)rows * TOPK_SLICES * SAMPLE_MAX_K);
        static TtbOncePerDevice configured;
        const size_t smem = (size_t)per * 8;
        if (configured.pending()) {
            cudaError_t e = cudaFuncSetAttribute(topk_slices_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 TOPK_MAX_SLICE * 8);
            if (e != cudaSuccess) return (int)e;
            configured.mark();
        }
        ttb_launch(topk_slices_kernel, dim3(TOPK_SLICES, rows), dim3(TOPK_THREADS), smem, stream, logits, ld, vocab,
                   temperature, top_k, cand, count);
        int status = ttb_launch_status();
        if (status != TTB_OK) return status;
        ttb_launch(topk_draw_kernel, dim3(rows), dim3(TOPK_THREADS), 0, stream, (const Cand*)cand, (const int*)count, vocab,
                   temperature, top_k, top_p, seeds, counters, out);
        status = ttb_launch_status();
        if (status != TTB_OK) return status;
    }
    ttb_launch(sample_kernel, rows, SAMPLE_THREADS, RADIX_BINS * sizeof(uint32_t), stream, logits, ld, vocab,
               temperature, top_k, top_p, seeds, counters, out, sliced ? 1 : 0);
    return ttb_launch_status();
}

TTB_EXPORT int ttb_sample_max_top_k() { return SAMPLE_MAX_K; }
TTB_EXPORT float ttb_sample_uniform(long long seed, int counter) {
    return uniform_from((uint64_t)seed, (uint64_t)(uint32_t)counter);
}
