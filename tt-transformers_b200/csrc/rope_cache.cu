// Rotation of queries and keys by their positions, fused with the write of keys and
// values into cache pages. Angles position * inv_freq, their sines and cosines and the
// rotation itself are float32; accurate sincosf (no fast-math).
//
// qkv row layout: [ heads * head_dim | kv_heads * head_dim | kv_heads * head_dim ].
// Rotation pairs element i with element i + rotary_dim/2 of each head, for i < rotary_dim/2
// (the checkpoint's row order), or, with `interleaved`, element 2i with element 2i + 1 (the
// order of models whose projections were trained on neighbouring pairs); elements from
// rotary_dim on are left as they are.
// Page layout: [num_pages, kv_heads, page_size, head_dim].
#include "common.cuh"

template <typename T, bool VEC>
__global__ void rope_kv_write_kernel(T* __restrict__ qkv, const int* __restrict__ positions,
                                     const int* __restrict__ seg_of_token, const float* __restrict__ inv_freq,
                                     int rotary_dim, int heads, int kv_heads, int head_dim,
                                     T* __restrict__ key_pages, T* __restrict__ value_pages,
                                     const int* __restrict__ block_table, int table_width, int page_size,
                                     int num_pages, int write_kv, int interleaved, int* __restrict__ status) {
    extern __shared__ float trig[];  // cos[rotary_dim/2], sin[rotary_dim/2]
    pdl_wait();
    pdl_launch_dependents();
    const int t = blockIdx.x;
    const int pos = positions[t];
    const int half_rot = rotary_dim / 2;
    for (int i = threadIdx.x; i < half_rot; i += blockDim.x) {
        const float angle = (float)pos * inv_freq[i];
        float s, c;
        sincosf(angle, &s, &c);
        trig[i] = c;
        trig[half_rot + i] = s;
    }
    __syncthreads();

    T* row = qkv + (size_t)t * (heads + 2 * kv_heads) * head_dim;
    const int half = head_dim / 2;

    if constexpr (VEC) {
        // Every pair of a head is rotated (rotary_dim == head_dim), head_dim is a multiple of 16 and rows and
        // pages are 16-byte aligned: a work item is eight consecutive elements i .. i+7 and their partners
        // i + half .., moved as two 16-byte words each way. Items: heads of q, then of k, then of v.
        constexpr int E = 16 / (int)sizeof(T);                  // elements in 16 bytes
        const int per_head = half / E;
        int page = -1, in_page = 0;
        if (write_kv) {
            const int page_index = pos / page_size;
            if (page_index >= table_width) {
                if (threadIdx.x == 0) atomicExch(status, 0x1000000 + t);
            } else {
                page = block_table[(size_t)seg_of_token[t] * table_width + page_index];
                if (page < 0 || page >= num_pages) {
                    if (threadIdx.x == 0) atomicExch(status, 0x2000000 + t);
                    page = -1;
                }
                in_page = pos - page_index * page_size;
            }
        }
        const int items = (heads + (write_kv ? 2 * kv_heads : 0)) * per_head;
        for (int w = threadIdx.x; w < items; w += blockDim.x) {
            const int h = w / per_head, i = (w - h * per_head) * E;      // h counts q heads, then k heads, then v heads
            const T* src = row + (size_t)h * head_dim;
            uint4 lo = *reinterpret_cast<const uint4*>(src + i), hi = *reinterpret_cast<const uint4*>(src + i + half);
            T* dst;
            if (h < heads) {
                dst = row + (size_t)h * head_dim;
            } else {
                if (page < 0) continue;
                const int g = (h - heads) % kv_heads;
                dst = (h - heads < kv_heads ? key_pages : value_pages) + (((size_t)page * kv_heads + g) * page_size + in_page) * head_dim;
            }
            if (h < heads + kv_heads) {                                   // queries and keys are rotated
                T* a = reinterpret_cast<T*>(&lo);
                T* b = reinterpret_cast<T*>(&hi);
#pragma unroll
                for (int e = 0; e < E; ++e) {
                    const float x = to_float(a[e]), y = to_float(b[e]);
                    const float c = trig[i + e], sn = trig[half_rot + i + e];
                    a[e] = from_float<T>(x * c - y * sn);
                    b[e] = from_float<T>(y * c + x * sn);
                }
            }
            *reinterpret_cast<uint4*>(dst + i) = lo;
            *reinterpret_cast<uint4*>(dst + i + half) = hi;
        }
    } else {
    // queries: rotate in place. Pair i is (i, i + half_rot), or (2i, 2i + 1) when interleaved.
    const int first = interleaved ? 2 : 1, apart = interleaved ? 1 : half_rot;
    for (int w = threadIdx.x; w < heads * half; w += blockDim.x) {
        const int h = w / half, i = w - h * half;
        if (i >= half_rot) continue;
        T* q = row + h * head_dim;
        const int ia = first * i, ib = ia + apart;
        const float a = to_float(q[ia]), b = to_float(q[ib]);
        const float c = trig[i], s = trig[half_rot + i];
        q[ia] = from_float<T>(a * c - b * s);
        q[ib] = from_float<T>(b * c + a * s);
    }
    if (!write_kv) return;

    const int page_index = pos / page_size;
    if (page_index >= table_width) {
        if (threadIdx.x == 0) atomicExch(status, 0x1000000 + t);
        return;
    }
    const int page = block_table[(size_t)seg_of_token[t] * table_width + page_index];
    if (page < 0 || page >= num_pages) {
        if (threadIdx.x == 0) atomicExch(status, 0x2000000 + t);
        return;
    }
    const int in_page = pos - page_index * page_size;
    const T* k_row = row + heads * head_dim;
    const T* v_row = k_row + kv_heads * head_dim;
    for (int w = threadIdx.x; w < kv_heads * half; w += blockDim.x) {
        const int g = w / half, i = w - g * half;
        const size_t dst = (((size_t)page * kv_heads + g) * page_size + in_page) * head_dim;
        const T* k = k_row + g * head_dim;
        const T* v = v_row + g * head_dim;
        // keys: element i pairs with i + half_rot when i < half_rot; the rest is copied.
        // Work item i covers elements i and i + half, so that every element is written once.
        if (i < half_rot) {
            const int ia = first * i, ib = ia + apart;
            const float a = to_float(k[ia]), b = to_float(k[ib]);
            const float c = trig[i], s = trig[half_rot + i];
            key_pages[dst + ia] = from_float<T>(a * c - b * s);
            key_pages[dst + ib] = from_float<T>(b * c + a * s);
        }
        value_pages[dst + i] = v[i];
        value_pages[dst + i + half] = v[i + half];
    }
    // key elements outside the rotated range [rotary_dim, head_dim) are copied unchanged
    if (rotary_dim < head_dim) {
        const int rest = head_dim - rotary_dim;
        for (int w = threadIdx.x; w < kv_heads * rest; w += blockDim.x) {
            const int g = w / rest, i = rotary_dim + (w - g * rest);
            const size_t dst = (((size_t)page * kv_heads + g) * page_size + in_page) * head_dim;
            key_pages[dst + i] = k_row[g * head_dim + i];
        }
    }
    }
}

TTB_EXPORT int ttb_rope_kv_write(void* qkv, int dtype, const int* positions, const int* seg_of_token,
                                 const float* inv_freq, int rotary_dim, int tokens, int heads, int kv_heads,
                                 int head_dim, void* key_pages, void* value_pages, const int* block_table,
                                 int table_width, int page_size, int num_pages, int write_kv, int interleaved,
                                 int* status, cudaStream_t stream) {
    if (tokens == 0) return TTB_OK;
    if (!qkv || !positions || !status) return TTB_ERR_ARGUMENT;
    if (write_kv && (!key_pages || !value_pages || !block_table || !seg_of_token)) return TTB_ERR_ARGUMENT;
    if (head_dim < 2 || (head_dim & 1)) return TTB_ERR_UNSUPPORTED;
    if (rotary_dim < 0 || rotary_dim > head_dim || (rotary_dim & 1)) return TTB_ERR_UNSUPPORTED;
    if (rotary_dim > 0 && !inv_freq) return TTB_ERR_ARGUMENT;
    const int threads = 256;
    const size_t smem = (size_t)(rotary_dim > 0 ? rotary_dim : 2) * sizeof(float);
    const int elem = dtype == TTB_DTYPE_BF16 ? 2 : 4;
    const bool vec = !interleaved && rotary_dim == head_dim && head_dim % (32 / elem) == 0 && aligned16(qkv) &&
                     (!write_kv || (aligned16(key_pages) && aligned16(value_pages)));
    if (vec && dtype == TTB_DTYPE_BF16)
        ttb_launch(rope_kv_write_kernel<__nv_bfloat16, true>, tokens, threads, smem, stream,
            (__nv_bfloat16*)qkv, positions, seg_of_token, inv_freq, rotary_dim, heads, kv_heads, head_dim,
            (__nv_bfloat16*)key_pages, (__nv_bfloat16*)value_pages, block_table, table_width, page_size, num_pages,
            write_kv, interleaved, status);
    else if (vec && dtype == TTB_DTYPE_F32)
        ttb_launch(rope_kv_write_kernel<float, true>, tokens, threads, smem, stream,
            (float*)qkv, positions, seg_of_token, inv_freq, rotary_dim, heads, kv_heads, head_dim,
            (float*)key_pages, (float*)value_pages, block_table, table_width, page_size, num_pages, write_kv, interleaved, status);
    else if (dtype == TTB_DTYPE_BF16)
        ttb_launch(rope_kv_write_kernel<__nv_bfloat16, false>, tokens, threads, smem, stream,
            (__nv_bfloat16*)qkv, positions, seg_of_token, inv_freq, rotary_dim, heads, kv_heads, head_dim,
            (__nv_bfloat16*)key_pages, (__nv_bfloat16*)value_pages, block_table, table_width, page_size, num_pages,
            write_kv, interleaved, status);
    else if (dtype == TTB_DTYPE_F32)
        ttb_launch(rope_kv_write_kernel<float, false>, tokens, threads, smem, stream,
            (float*)qkv, positions, seg_of_token, inv_freq, rotary_dim, heads, kv_heads, head_dim,
            (float*)key_pages, (float*)value_pages, block_table, table_width, page_size, num_pages, write_kv, interleaved, status);
    else
        return TTB_ERR_UNSUPPORTED;
    return ttb_launch_status();
}
