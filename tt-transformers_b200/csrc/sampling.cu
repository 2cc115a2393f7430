// Token selection from float32 logits, one block per row.
//   temperature == 0          the largest logit; among equal ones the lowest token id.
//   temperature > 0           softmax(logits / temperature) in float32 and an inverse-CDF draw
//                             with u in [0, 1) taken from (seed, counter) alone, so that a
//                             request's stream does not depend on its place in the batch.
//   top_k in 1..SAMPLE_MAX_K  only the k largest logits take part (lowest id first among equal
//                             ones); they are walked from the largest down.
//   top_p < 1                 of those, the low tail whose cumulative probability is <= 1 - top_p
//                             is left out; the largest always stays.
//   top_k > SAMPLE_MAX_K, or top_p < 1 without top_k: the cuts are found as thresholds on the logit's
//                             value, by bisection over its 32 bits (no sorting): first the value of
//                             the k-th largest logit, everything below it is out; then the largest
//                             value t such that the logits below t (of those still in) hold at most
//                             1 - top_p of the probability, and everything below t is out. Logits
//                             equal to a threshold all stay. The draw walks the vocabulary in id order.
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

__global__ void __launch_bounds__(SAMPLE_THREADS)
sample_kernel(const float* __restrict__ logits, int ld, int vocab, const float* __restrict__ temperature,
              const int* __restrict__ top_k, const float* __restrict__ top_p, const long long* __restrict__ seeds,
              const int* __restrict__ counters, int* __restrict__ out) {
    __shared__ Best best_scratch[32];
    __shared__ float sum_scratch[32];
    __shared__ float chunk_sum[SAMPLE_THREADS];
    __shared__ float cand_value[SAMPLE_MAX_K];
    __shared__ int cand_index[SAMPLE_MAX_K];
    __shared__ int result;
    pdl_wait();
    pdl_launch_dependents();
    const int row = blockIdx.x;
    const float* l = logits + (size_t)row * ld;
    const int tid = threadIdx.x;

    Best mine{-INFINITY, 0x7fffffff};
    for (int i = tid; i < vocab; i += SAMPLE_THREADS) mine = better(mine, Best{l[i], i});
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
        if (k > SAMPLE_MAX_K && k < vocab) {
            // the key of the k-th largest logit: the largest key with at least k logits at or above it
            uint32_t prefix = 0;
            for (int bit = 31; bit >= 0; --bit) {
                const uint32_t candidate = prefix | (1u << bit);
                float count = 0.f;                       // exact in float up to 2^24 entries per row
                for (int i = tid; i < vocab; i += SAMPLE_THREADS) count += ordered_key(l[i]) >= candidate ? 1.f : 0.f;
                count = block_sum(count, sum_scratch);
                if (count >= (float)k) prefix = candidate;
            }
            cut = prefix;
        }
        if (p_limit < 1.f) {
            float kept = 0.f;
            for (int i = tid; i < vocab; i += SAMPLE_THREADS)
                if (ordered_key(l[i]) >= cut) kept += expf((l[i] - top.value) * inv_temp);
            kept = block_sum(kept, sum_scratch);
            const float limit = (1.f - p_limit) * kept;
            // the largest key t with mass{cut <= key < t} <= limit; logits below t leave
            uint32_t prefix = 0;
            for (int bit = 31; bit >= 0; --bit) {
                const uint32_t candidate = prefix | (1u << bit);
                float below = 0.f;
                if (candidate > cut) {
                    for (int i = tid; i < vocab; i += SAMPLE_THREADS) {
                        const uint32_t key = ordered_key(l[i]);
                        if (key >= cut && key < candidate) below += expf((l[i] - top.value) * inv_temp);
                    }
                }
                below = block_sum(below, sum_scratch);
                if (below <= limit) prefix = candidate;
            }
            cut = prefix < top_key ? prefix : top_key;   // the largest logit always stays
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

TTB_EXPORT int ttb_sample(const float* logits, int ld, int rows, int vocab, const float* temperature,
                          const int* top_k, const float* top_p, const long long* seeds, const int* counters,
                          int* out, cudaStream_t stream) {
    if (rows == 0) return TTB_OK;
    if (!logits || !out || vocab < 1) return TTB_ERR_ARGUMENT;
    if (temperature && (!seeds || !counters)) return TTB_ERR_ARGUMENT;
    ttb_launch(sample_kernel, rows, SAMPLE_THREADS, 0, stream, logits, ld, vocab, temperature, top_k, top_p, seeds, counters, out);
    return ttb_launch_status();
}

TTB_EXPORT int ttb_sample_max_top_k() { return SAMPLE_MAX_K; }
TTB_EXPORT float ttb_sample_uniform(long long seed, int counter) {
    return uniform_from((uint64_t)seed, (uint64_t)(uint32_t)counter);
}
