// Embedding lookup, residual add + RMSNorm, SwiGLU gate, row gather.
// The residual stream is float32 in every precision; the sum, the mean of squares
// and the scaling are computed in float32.
#include "common.cuh"

// ---------------------------------------------------------------- embedding: out[t, :] = table[ids[t], :] as float32
template <typename T>
__global__ void embedding_kernel(const T* __restrict__ table, const int* __restrict__ ids, float* __restrict__ out,
                                 int width, int vocab, float scale, int* __restrict__ status) {
    pdl_wait();
    pdl_launch_dependents();
    const int t = blockIdx.x;
    const int id = ids[t];
    if (id < 0 || id >= vocab) {              // never read outside the table: flag it, write zeros
        if (threadIdx.x == 0) atomicExch(status, 1 + t);
        for (int c = threadIdx.x; c < width; c += blockDim.x) out[(size_t)t * width + c] = 0.f;
        return;
    }
    const T* row = table + (size_t)id * width;
    float* dst = out + (size_t)t * width;
    if ((width & 7) == 0) {
        for (int c = threadIdx.x * 8; c < width; c += blockDim.x * 8) {
            float v[8];
            load8(row + c, v);
            if (scale != 1.f) {
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] *= scale;
            }
            store8(dst + c, v);
        }
    } else {
        for (int c = threadIdx.x; c < width; c += blockDim.x) dst[c] = to_float(row[c]) * scale;
    }
}

// scale: every embedded row is multiplied by it in float32 (1 for none).
TTB_EXPORT int ttb_embedding(const void* table, int dtype, const int* ids, float* out, int tokens, int width,
                             int vocab, float scale, int* status, cudaStream_t stream) {
    if (tokens == 0) return TTB_OK;
    if (!table || !ids || !out || !status) return TTB_ERR_ARGUMENT;
    if (!aligned16(table) || !aligned16(out)) return TTB_ERR_ARGUMENT;
    const int threads = 128;
    if (dtype == TTB_DTYPE_BF16)
        ttb_launch(embedding_kernel<__nv_bfloat16>, tokens, threads, 0, stream, (const __nv_bfloat16*)table, ids, out, width, vocab, scale, status);
    else if (dtype == TTB_DTYPE_F32)
        ttb_launch(embedding_kernel<float>, tokens, threads, 0, stream, (const float*)table, ids, out, width, vocab, scale, status);
    else
        return TTB_ERR_UNSUPPORTED;
    return ttb_launch_status();
}

// ---------------------------------------------------------------- residual += delta; out = rmsnorm(residual) * w
// One block per row. The summed row is kept in shared memory between the two passes.
template <typename TD, typename TW, typename TO, bool VEC>
__global__ void add_rmsnorm_kernel(float* __restrict__ residual, const TD* __restrict__ delta,
                                   const TW* __restrict__ weight, TO* __restrict__ out, int width, float eps) {
    extern __shared__ float row[];
    __shared__ float scratch[32];
    const size_t base = (size_t)blockIdx.x * width;
    if (VEC && width <= (int)blockDim.x * 8) {
        // A row in one pass (decode: a handful of rows, every microsecond of this kernel is on the step's
        // critical path): the thread's eight values stay in registers, and the norm's weight, which no
        // kernel writes, is fetched before the wait for the kernel before this one.
        const int c = threadIdx.x * 8;
        const bool mine = c < width;
        float w[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (mine) load8(weight + c, w);
        pdl_wait();
        pdl_launch_dependents();
        float sumsq = 0.f;
        if (mine) {
            load8(residual + base + c, v);
            if (delta != nullptr) {
                float d[8];
                load8(delta + base + c, d);
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] += d[e];
                store8(residual + base + c, v);
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) sumsq += v[e] * v[e];
        }
        sumsq = block_sum(sumsq, scratch);
        const float scale = rsqrtf(sumsq / (float)width + eps);
        if (mine) {
            float o[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = v[e] * scale * w[e];
            store8(out + base + c, o);
        }
        return;
    }
    pdl_wait();
    pdl_launch_dependents();
    float sumsq = 0.f;
    if (VEC) {      // width a multiple of 8, all pointers 16-byte aligned: eight elements per thread and pass
        for (int c = threadIdx.x * 8; c < width; c += blockDim.x * 8) {
            float v[8];
            load8(residual + base + c, v);
            if (delta != nullptr) {
                float d[8];
                load8(delta + base + c, d);
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] += d[e];
                store8(residual + base + c, v);
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                row[c + e] = v[e];
                sumsq += v[e] * v[e];
            }
        }
    } else {
        for (int c = threadIdx.x; c < width; c += blockDim.x) {
            float v = residual[base + c];
            if (delta != nullptr) {
                v += to_float(delta[base + c]);
                residual[base + c] = v;
            }
            row[c] = v;
            sumsq += v * v;
        }
    }
    sumsq = block_sum(sumsq, scratch);
    const float scale = rsqrtf(sumsq / (float)width + eps);
    if (VEC) {
        for (int c = threadIdx.x * 8; c < width; c += blockDim.x * 8) {
            float w[8], o[8];
            load8(weight + c, w);
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = row[c + e] * scale * w[e];
            store8(out + base + c, o);
        }
    } else {
        for (int c = threadIdx.x; c < width; c += blockDim.x)
            out[base + c] = from_float<TO>(row[c] * scale * to_float(weight[c]));
    }
}

template <typename TD, typename TO>
static int launch_add_rmsnorm(float* residual, const void* delta, const void* weight, int weight_dtype, void* out,
                              int rows, int width, float eps, cudaStream_t stream) {
    const size_t smem = (size_t)width * sizeof(float);
    const bool vec = (width % 8 == 0) && aligned16(residual) && aligned16(weight) && aligned16(out) &&
                     (delta == nullptr || aligned16(delta));
    const int per_thread = vec ? 8 : 1;
    const int want = (width + per_thread - 1) / per_thread;
    const int threads = want >= 512 ? 512 : (want >= 256 ? 256 : (want >= 128 ? 128 : 64));
#define NORM_LAUNCH(TW, V)                                                                                     \
    do {                                                                                                       \
        auto k = add_rmsnorm_kernel<TD, TW, TO, V>;                                                            \
        if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
        ttb_launch(k, rows, threads, smem, stream, residual, (const TD*)delta, (const TW*)weight, (TO*)out, width, eps); \
    } while (0)
    if (weight_dtype == TTB_DTYPE_F32) {
        if (vec) NORM_LAUNCH(float, true); else NORM_LAUNCH(float, false);
    } else {
        if (vec) NORM_LAUNCH(__nv_bfloat16, true); else NORM_LAUNCH(__nv_bfloat16, false);
    }
#undef NORM_LAUNCH
    return ttb_launch_status();
}

// dtype: type of delta and out (the compute dtype). weight_dtype may differ (a weight stored in 32-bit stays so).
TTB_EXPORT int ttb_add_rmsnorm(float* residual, const void* delta, const void* weight, int weight_dtype, void* out,
                               int dtype, int rows, int width, float eps, cudaStream_t stream) {
    if (rows == 0) return TTB_OK;
    if (!residual || !weight || !out) return TTB_ERR_ARGUMENT;
    if ((size_t)width * sizeof(float) > 200 * 1024) return TTB_ERR_UNSUPPORTED;  // row must fit shared memory
    if (weight_dtype != TTB_DTYPE_F32 && weight_dtype != TTB_DTYPE_BF16) return TTB_ERR_UNSUPPORTED;
    if (dtype == TTB_DTYPE_BF16)
        return launch_add_rmsnorm<__nv_bfloat16, __nv_bfloat16>(residual, delta, weight, weight_dtype, out, rows, width, eps, stream);
    if (dtype == TTB_DTYPE_F32)
        return launch_add_rmsnorm<float, float>(residual, delta, weight, weight_dtype, out, rows, width, eps, stream);
    return TTB_ERR_UNSUPPORTED;
}

// ---------------------------------------------------------------- out[t, i] = silu(gate_up[t, i]) * gate_up[t, I + i]
template <typename T, bool VEC>
__global__ void swiglu_kernel(const T* __restrict__ gate_up, T* __restrict__ out, int rows, int inter) {
    pdl_wait();
    pdl_launch_dependents();
    if (VEC) {      // inter a multiple of 8 and 16-byte aligned bases: eight outputs per thread
        const int per_row = inter / 8;
        const size_t total = (size_t)rows * per_row;
        for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (size_t)gridDim.x * blockDim.x) {
            const size_t t = idx / per_row;
            const int i = (int)(idx - t * per_row) * 8;
            float g[8], u[8], o[8];
            load8(gate_up + t * 2 * inter + i, g);
            load8(gate_up + t * 2 * inter + inter + i, u);
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = g[e] / (1.f + expf(-g[e])) * u[e];
            store8(out + t * inter + i, o);
        }
        return;
    }
    const size_t total = (size_t)rows * inter;
    for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (size_t)gridDim.x * blockDim.x) {
        const size_t t = idx / inter;
        const int i = (int)(idx - t * inter);
        const float g = to_float(gate_up[t * 2 * inter + i]);
        const float u = to_float(gate_up[t * 2 * inter + inter + i]);
        const float s = g / (1.f + expf(-g));
        out[idx] = from_float<T>(s * u);
    }
}

TTB_EXPORT int ttb_swiglu(const void* gate_up, void* out, int dtype, int rows, int inter, cudaStream_t stream) {
    if (rows == 0) return TTB_OK;
    if (!gate_up || !out) return TTB_ERR_ARGUMENT;
    const bool vec = (inter % 8 == 0) && aligned16(gate_up) && aligned16(out);
    const size_t total = (size_t)rows * (vec ? inter / 8 : inter);
    const int threads = 256;
    const size_t want = (total + threads - 1) / threads;
    const int blocks = (int)(want < 148 * 32 ? want : 148 * 32);
    if (dtype == TTB_DTYPE_BF16) {
        if (vec) ttb_launch(swiglu_kernel<__nv_bfloat16, true>, blocks, threads, 0, stream, (const __nv_bfloat16*)gate_up, (__nv_bfloat16*)out, rows, inter);
        else ttb_launch(swiglu_kernel<__nv_bfloat16, false>, blocks, threads, 0, stream, (const __nv_bfloat16*)gate_up, (__nv_bfloat16*)out, rows, inter);
    } else if (dtype == TTB_DTYPE_F32) {
        if (vec) ttb_launch(swiglu_kernel<float, true>, blocks, threads, 0, stream, (const float*)gate_up, (float*)out, rows, inter);
        else ttb_launch(swiglu_kernel<float, false>, blocks, threads, 0, stream, (const float*)gate_up, (float*)out, rows, inter);
    } else {
        return TTB_ERR_UNSUPPORTED;
    }
    return ttb_launch_status();
}

// ---------------------------------------------------------------- dst[n, :] = src[rows[n], :], rows of row_bytes bytes
template <typename U>
__global__ void gather_rows_kernel(const U* __restrict__ src, const int* __restrict__ rows, U* __restrict__ dst,
                                   int units_per_row) {
    pdl_wait();
    pdl_launch_dependents();
    const U* s = src + (size_t)rows[blockIdx.x] * units_per_row;
    U* d = dst + (size_t)blockIdx.x * units_per_row;
    for (int c = threadIdx.x; c < units_per_row; c += blockDim.x) d[c] = s[c];
}

TTB_EXPORT int ttb_gather_rows(const void* src, const int* rows, void* dst, int count, int row_bytes,
                               cudaStream_t stream) {
    if (count == 0) return TTB_OK;
    if (!src || !rows || !dst) return TTB_ERR_ARGUMENT;
    const int threads = 128;
    if ((row_bytes & 15) == 0 && aligned16(src) && aligned16(dst))
        ttb_launch(gather_rows_kernel<uint4>, count, threads, 0, stream, (const uint4*)src, rows, (uint4*)dst, row_bytes / 16);
    else if ((row_bytes & 3) == 0)
        ttb_launch(gather_rows_kernel<uint32_t>, count, threads, 0, stream, (const uint32_t*)src, rows, (uint32_t*)dst, row_bytes / 4);
    else if ((row_bytes & 1) == 0)
        ttb_launch(gather_rows_kernel<uint16_t>, count, threads, 0, stream, (const uint16_t*)src, rows, (uint16_t*)dst, row_bytes / 2);
    else
        return TTB_ERR_UNSUPPORTED;
    return ttb_launch_status();
}

// ---------------------------------------------------------------- x = cap * tanh(x / cap), float32, in place
// A capped head: logits are squashed into (-cap, cap). Rows are `stride` floats apart.
__global__ void softcap_kernel(float* __restrict__ x, int cols, int stride, float cap) {
    pdl_wait();
    pdl_launch_dependents();
    float* row = x + (size_t)blockIdx.y * stride;
    const float inv = 1.f / cap;
    for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < cols; c += gridDim.x * blockDim.x)
        row[c] = cap * tanhf(row[c] * inv);
}

TTB_EXPORT int ttb_softcap(float* x, int rows, int cols, int stride, float cap, cudaStream_t stream) {
    if (rows == 0 || cols == 0) return TTB_OK;
    if (!x || !(cap > 0.f) || stride < cols) return TTB_ERR_ARGUMENT;
    if (rows > 65535) return TTB_ERR_UNSUPPORTED;
    const int threads = 256;
    int bx = (cols + threads - 1) / threads;
    if (bx > 64) bx = 64;
    ttb_launch(softcap_kernel, dim3(bx, rows), threads, 0, stream, x, cols, stride, cap);
    return ttb_launch_status();
}
