// Weight-streaming matrix product for decoding on the tensor cores:
//   out[m, n] = sum_k x[m, k] * w[n, k]     for M <= 64 rows of x (one per decoded token).
// The weight matrix is the 16-row operand of mma.m16n8k16 and the activations the 8-column one,
// so a handful of tokens costs no more tensor work than one. Every weight is read from HBM
// once, with 16-byte loads that go straight into the fragment registers: within a block of 32
// k, lane t of a quad holds k = 8t .. 8t+7 for both operands, which is a permutation of k that
// the sum does not see. The 8 or 16 warps of a block share the same weight rows and take the
// k-blocks in turn, several blocks of loads in flight each; their partial sums meet in shared
// memory. Matrices with few rows and a long K get 16 warps: with few blocks per SM, the bytes in
// flight per block decide the bandwidth.
//
// Row modes of a 16-row fragment:
//   FULL  rows n0 .. n0+15 of w
//   HALF  rows n0 .. n0+7 of w, upper half zero (more blocks for matrices with few rows)
//   PAIR  rows n0 .. n0+7 of w (gate) and of w + pair_offset rows (up); the epilogue writes
//         silu(gate) * up, so the SwiGLU product never round-trips through memory
//   ROPE  the fused QKV projection of a decode step: a block owns rows i .. i+7 of one head and their
//         rotation partners i + head_dim/2 .., so that the epilogue can rotate query and key pairs by
//         their positions (float32 angles, accurate sincosf), write the queries out and put keys and
//         values straight into their cache pages; no rotation kernel and no qkv round trip
//
// Two fusions with the steps around the product take the norm kernel out of a decode layer. The
// product that ends a sub-layer (`residual` set) adds its result to the float32 residual stream in
// place, writes xg = bfloat16(g * residual), g being the weight of the norm that follows, and leaves
// the sum of residual^2 over its rows of every token in ssq_out[block]. The product that begins the
// next sub-layer (NORM) takes xg as its x, adds the partial sums up and scales its results by
// 1 / sqrt(sum / K + eps):  W (g * r / rms(r)) = (W (g * r)) / rms(r). Every element of the stream
// belongs to one thread of one block, and the partial sums are added in a fixed order, so the
// result does not change from run to run.
#include "common.cuh"

#define GM_FULL 0
#define GM_HALF 1
#define GM_PAIR 2
#define GM_ROPE 3

// What the fused QKV mode needs beyond the product: positions, rotation frequencies and the cache.
struct GmRope {
    const int* positions;        // [M]
    const int* seg_of_token;     // [M]
    const float* inv_freq;       // [head_dim / 2]
    const int* block_table;      // [segments, table_width]
    __nv_bfloat16* key_pages;    // [num_pages, kv_heads, page_size, head_dim]
    __nv_bfloat16* value_pages;
    int* status;
    int table_width, page_size, num_pages, heads, kv_heads, head_dim, write_kv;
};

// The fusions' operands (null / 0 when unused).
struct GmFuse {
    // the product that begins a sub-layer: x = g * residual, to be divided by the rows' RMS
    const float* ssq_in;         // [ssq_parts][16] partial sums of residual^2 per token
    int ssq_parts;
    float eps;
    // the product that ends a sub-layer
    float* residual;             // [M, ldr] float32: the product is added here
    int ldr;
    const float* next_weight;    // [N] float32 weight of the norm that follows (null: only the add)
    __nv_bfloat16* xg;           // [M, ldxg] = bfloat16(next_weight * residual)
    int ldxg;
    float* ssq_out;              // [blocks][16]
};

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ uint4 ldg_cached(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ACCUM (the epilogue that adds to the residual stream) is a template parameter and not a test of
// `fuse.residual`: with that epilogue compiled in, the plain 8-row shapes came out with 58 registers
// a thread instead of 32, and although the product by itself got faster, the decode step got slower
// (fewer blocks of the kernels before and after fit beside them while those start early and wait).
template <int NB, int RG, int MODE, int GM_WARPS, typename TO, bool NORM, bool ACCUM>
__global__ void __launch_bounds__(GM_WARPS * 32)
gemv_mma_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w, TO* __restrict__ out,
                int M, int N, int K, int ldx, int ldw, int ldo, int pair_offset, GmRope rope, GmFuse fuse) {
    constexpr int ROWS_PER_GROUP = (MODE == GM_FULL) ? 16 : 8;
    constexpr int GM_THREADS = GM_WARPS * 32;
    extern __shared__ float4 partial[];          // [GM_WARPS][RG * NB * 32], then (NORM) float [GM_WARPS * 2][16] sums of squares
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    int n0 = blockIdx.x * ROWS_PER_GROUP * RG;
    if (MODE == GM_ROPE) {       // blocks per head: head_dim / 16; eight rows of the first half, pair_offset = head_dim / 2
        const int per_head = rope.head_dim >> 4;
        n0 = (blockIdx.x / per_head) * rope.head_dim + (blockIdx.x % per_head) * 8;
    }

    // row pointers of this thread: [rg][half]
    const __nv_bfloat16* wrow[RG][2];
#pragma unroll
    for (int rg = 0; rg < RG; ++rg) {
        int lower = n0 + rg * ROWS_PER_GROUP + g;
        if (lower > N - 1) lower = N - 1;                       // clamped rows are computed and not written
        wrow[rg][0] = w + (size_t)lower * ldw;
        if (MODE == GM_FULL) {
            int upper = n0 + rg * 16 + 8 + g;
            if (upper > N - 1) upper = N - 1;
            wrow[rg][1] = w + (size_t)upper * ldw;
        } else if (MODE == GM_PAIR || MODE == GM_ROPE) {
            wrow[rg][1] = w + (size_t)(lower + pair_offset) * ldw;
        } else {
            wrow[rg][1] = nullptr;
        }
    }
    // The weights do not depend on the kernels before this one: ask L2 for this block's rows now,
    // then wait for the predecessor (whose output is x). (Loading the first k-blocks into registers
    // here instead made a chain of products faster and the whole decode step slower: the loads of
    // blocks that wait compete with the kernel that the step is waiting for.)
    pdl_launch_dependents();
    {
        const int row_bytes = K * 2;
        const int lines = (row_bytes + 127) / 128;
        constexpr int HALVES = (MODE == GM_HALF) ? 1 : 2;
        for (int i = threadIdx.x; i < RG * HALVES * 8 * lines; i += GM_THREADS) {
            const int line = i % lines, r = i / lines;                 // r: (rg, half, row of eight)
            const int rg = r / (HALVES * 8), h = (r / 8) % HALVES, gg = r % 8;
            int lower = n0 + rg * ROWS_PER_GROUP + gg;
            if (lower > N - 1) lower = N - 1;
            int row = lower;
            if (h == 1) row = (MODE == GM_FULL) ? min(n0 + rg * 16 + 8 + gg, N - 1) : lower + pair_offset;
            const char* p = reinterpret_cast<const char*>(w + (size_t)row * ldw) + (size_t)line * 128;
            asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
        }
    }
    pdl_wait();
    // NORM: thread `tid` adds up the partial sums of token tid % 16 over the parts tid / 16, tid / 16 + threads / 16, ...
    float ssq_mine = 0.f;
    if (NORM) {
        for (int p = threadIdx.x >> 4; p < fuse.ssq_parts; p += GM_THREADS >> 4) ssq_mine += fuse.ssq_in[p * 16 + (threadIdx.x & 15)];
    }
    const __nv_bfloat16* xrow[NB];
    bool xok[NB];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
        const int m = nb * 8 + g;
        xok[nb] = m < M;
        xrow[nb] = x + (size_t)(xok[nb] ? m : 0) * ldx;
    }

    float acc[RG][NB][4];
#pragma unroll
    for (int rg = 0; rg < RG; ++rg)
#pragma unroll
        for (int nb = 0; nb < NB; ++nb)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[rg][nb][c] = 0.f;

    const uint4 zero = make_uint4(0, 0, 0, 0);
    constexpr int UNROLL = (RG * NB >= 8) ? 2 : (RG * NB >= 2 ? 4 : 8);
    // warp `warp` takes the k-blocks warp, warp + GM_WARPS, ... ; UNROLL of them are in flight at a time
    for (int kb0 = warp * 32; kb0 < K; kb0 += GM_WARPS * 32 * UNROLL) {
        uint4 wv[UNROLL][RG][2];
        uint4 xv[UNROLL][NB];
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            const int k = kb0 + u * GM_WARPS * 32 + t * 8;
            const bool in = k < K;
#pragma unroll
            for (int rg = 0; rg < RG; ++rg) {
                wv[u][rg][0] = in ? ldg_stream(wrow[rg][0] + k) : zero;
                wv[u][rg][1] = (in && MODE != GM_HALF) ? ldg_stream(wrow[rg][1] + k) : zero;
            }
#pragma unroll
            for (int nb = 0; nb < NB; ++nb) xv[u][nb] = (in && xok[nb]) ? ldg_cached(xrow[nb] + k) : zero;
        }
#pragma unroll
        for (int u = 0; u < UNROLL; ++u)
#pragma unroll
            for (int rg = 0; rg < RG; ++rg)
#pragma unroll
                for (int nb = 0; nb < NB; ++nb) {
                    mma16816(acc[rg][nb], wv[u][rg][0].x, wv[u][rg][1].x, wv[u][rg][0].y, wv[u][rg][1].y,
                             xv[u][nb].x, xv[u][nb].y);
                    mma16816(acc[rg][nb], wv[u][rg][0].z, wv[u][rg][1].z, wv[u][rg][0].w, wv[u][rg][1].w,
                             xv[u][nb].z, xv[u][nb].w);
                }
    }

    // ---- the warps add up
    constexpr int PER_WARP = RG * NB * 32;
#pragma unroll
    for (int rg = 0; rg < RG; ++rg)
#pragma unroll
        for (int nb = 0; nb < NB; ++nb)
            partial[warp * PER_WARP + (rg * NB + nb) * 32 + lane] =
                make_float4(acc[rg][nb][0], acc[rg][nb][1], acc[rg][nb][2], acc[rg][nb][3]);
    float* ssq_groups = reinterpret_cast<float*>(partial + GM_WARPS * PER_WARP);     // [GM_THREADS / 16][16]
    if (NORM) ssq_groups[threadIdx.x] = ssq_mine;
    __syncthreads();
    for (int e = threadIdx.x; e < PER_WARP; e += GM_THREADS) {
        float4 s = partial[e];
#pragma unroll
        for (int wp = 1; wp < GM_WARPS; ++wp) {
            const float4 p = partial[wp * PER_WARP + e];
            s.x += p.x; s.y += p.y; s.z += p.z; s.w += p.w;
        }
        const int el = e & 31, nb = (e >> 5) % NB, rg = (e >> 5) / NB;
        const int eg = el >> 2, et = el & 3;
        const int m0 = nb * 8 + 2 * et, m1 = m0 + 1;
        const int lower = n0 + rg * ROWS_PER_GROUP + eg;
        if (NORM) {
            float q0 = 0.f, q1 = 0.f;
#pragma unroll
            for (int grp = 0; grp < (GM_THREADS >> 4); ++grp) {        // the same order in every block and on every run
                q0 += ssq_groups[grp * 16 + (m0 & 15)];
                q1 += ssq_groups[grp * 16 + (m1 & 15)];
            }
            const float r0 = rsqrtf(q0 / (float)K + fuse.eps), r1 = rsqrtf(q1 / (float)K + fuse.eps);
            s.x *= r0; s.z *= r0;
            s.y *= r1; s.w *= r1;
        }
        if (MODE == GM_ROPE) {
            const int hd = rope.head_dim, half = hd >> 1;
            const int head = lower / hd, i = lower - head * hd;             // i < half: index of the rotation pair
            const bool is_q = head < rope.heads, is_k = !is_q && head < rope.heads + rope.kv_heads;
            const float freq = (is_q || is_k) ? rope.inv_freq[i] : 0.f;
#pragma unroll
            for (int which = 0; which < 2; ++which) {
                const int m = which ? m1 : m0;
                if (m >= M) continue;
                float lo = which ? s.y : s.x, up = which ? s.w : s.z;
                const int pos = rope.positions[m];
                if (is_q || is_k) {
                    float sn, cs;
                    sincosf((float)pos * freq, &sn, &cs);
                    const float a = lo, b = up;
                    lo = a * cs - b * sn;
                    up = b * cs + a * sn;
                }
                if (is_q) {
                    out[(size_t)m * ldo + lower] = from_float<TO>(lo);
                    out[(size_t)m * ldo + lower + half] = from_float<TO>(up);
                } else if (rope.write_kv) {
                    const int kvh = head - rope.heads - (is_k ? 0 : rope.kv_heads);
                    const int page_index = pos / rope.page_size;
                    int page = -1;
                    if (page_index < rope.table_width)
                        page = rope.block_table[(size_t)rope.seg_of_token[m] * rope.table_width + page_index];
                    if ((unsigned)page >= (unsigned)rope.num_pages) {
                        atomicExch(rope.status, 0x2000000 + m);              // outside the pool: skip the write, say so
                    } else {
                        __nv_bfloat16* dst = (is_k ? rope.key_pages : rope.value_pages) +
                            (((size_t)page * rope.kv_heads + kvh) * rope.page_size + (pos - page_index * rope.page_size)) * hd;
                        dst[i] = __float2bfloat16_rn(lo);
                        dst[i + half] = __float2bfloat16_rn(up);
                    }
                }
            }
        } else if (MODE == GM_PAIR) {
            if (lower < N) {
                if (m0 < M) out[(size_t)m0 * ldo + lower] = from_float<TO>(s.x / (1.f + __expf(-s.x)) * s.z);
                if (m1 < M) out[(size_t)m1 * ldo + lower] = from_float<TO>(s.y / (1.f + __expf(-s.y)) * s.w);
            }
        } else if (ACCUM) {
            // the end of a sub-layer: add to the stream; for the norm that follows, g * stream and the rows' squares
            const int upper = n0 + rg * 16 + 8 + eg;
            float q0 = 0.f, q1 = 0.f;
#pragma unroll
            for (int which = 0; which < 4; ++which) {
                const int m = (which & 1) ? m1 : m0, n = (which & 2) ? upper : lower;
                if ((which & 2) && MODE != GM_FULL) continue;
                if (m >= M || n >= N) continue;
                const float delta = which == 0 ? s.x : which == 1 ? s.y : which == 2 ? s.z : s.w;
                float* at = fuse.residual + (size_t)m * fuse.ldr + n;
                const float r = *at + delta;
                *at = r;
                if (fuse.xg != nullptr) {
                    fuse.xg[(size_t)m * fuse.ldxg + n] = __float2bfloat16_rn(r * fuse.next_weight[n]);
                    if (which & 1) q1 += r * r; else q0 += r * r;
                }
            }
            if (fuse.xg != nullptr) {      // whole warps are here (RG = 1): lanes that differ in eg hold different rows of w
#pragma unroll
                for (int o = 4; o < 32; o <<= 1) {
                    q0 += __shfl_xor_sync(0xffffffffu, q0, o);
                    q1 += __shfl_xor_sync(0xffffffffu, q1, o);
                }
                if (eg == 0) {
                    fuse.ssq_out[(size_t)blockIdx.x * 16 + (m0 & 15)] = q0;
                    fuse.ssq_out[(size_t)blockIdx.x * 16 + (m1 & 15)] = q1;
                }
            }
        } else {
            if (lower < N) {
                if (m0 < M) out[(size_t)m0 * ldo + lower] = from_float<TO>(s.x);
                if (m1 < M) out[(size_t)m1 * ldo + lower] = from_float<TO>(s.y);
            }
            if (MODE == GM_FULL) {
                const int upper = n0 + rg * 16 + 8 + eg;
                if (upper < N) {
                    if (m0 < M) out[(size_t)m0 * ldo + upper] = from_float<TO>(s.z);
                    if (m1 < M) out[(size_t)m1 * ldo + upper] = from_float<TO>(s.w);
                }
            }
        }
    }
}

template <int NB, int RG, int MODE, int GM_WARPS, typename TO, bool NORM = false, bool ACCUM = false>
static int gemv_mma_launch(const void* x, const void* w, void* out, int M, int N, int K, int ldx, int ldw, int ldo,
                           int pair_offset, cudaStream_t stream, const GmRope* rope = nullptr,
                           const GmFuse* fuse = nullptr) {
    constexpr int rows = ((MODE == GM_FULL) ? 16 : 8) * RG;
    constexpr int GM_THREADS = GM_WARPS * 32;
    const size_t smem = (size_t)GM_WARPS * RG * NB * 32 * sizeof(float4) + (NORM ? (size_t)GM_THREADS * sizeof(float) : 0);
    auto kernel = gemv_mma_kernel<NB, RG, MODE, GM_WARPS, TO, NORM, ACCUM>;
    static TtbOncePerDevice configured;
    if (configured.pending() && smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return (int)e;
    }
    configured.mark();
    GmRope none = {};
    GmFuse plain = {};
    const int blocks = (MODE == GM_ROPE) ? N / 16 : (N + rows - 1) / rows;
    ttb_launch(kernel, dim3(blocks), dim3(GM_THREADS), smem, stream,
        (const __nv_bfloat16*)x, (const __nv_bfloat16*)w, (TO*)out, M, N, K, ldx, ldw, ldo, pair_offset,
        rope ? *rope : none, fuse ? *fuse : plain);
    return ttb_launch_status();
}

// few blocks and a long K: sixteen warps per block keep enough loads in flight
static bool gemv_mma_wide(int N, int K, int rows_small) { return K >= 4096 && (N + rows_small - 1) / rows_small < 4 * 148; }
// matrices with few rows get 8-row fragments, so that there are blocks enough for every SM
static bool gemv_mma_half(int M, int N) { return (N / 16) < 2 * 148 && M <= 32; }

template <int MODE, typename TO, bool NORM = false, bool ACCUM = false>
static int gemv_mma_by_rows(const void* x, const void* w, void* out, int M, int N, int K, int ldx, int ldw, int ldo,
                            int pair_offset, cudaStream_t stream, const GmFuse* fuse = nullptr) {
    constexpr int rows_small = (MODE == GM_FULL) ? 16 : 8;
    const bool wide = gemv_mma_wide(N, K, rows_small);
#define GM_GO(NB, RG)                                                                                                      \
    do {                                                                                                                   \
        if (wide)                                                                                                          \
            return gemv_mma_launch<NB, RG, MODE, 16, TO, NORM, ACCUM>(x, w, out, M, N, K, ldx, ldw, ldo, pair_offset,      \
                                                                      stream, nullptr, fuse);                              \
        return gemv_mma_launch<NB, RG, MODE, 8, TO, NORM, ACCUM>(x, w, out, M, N, K, ldx, ldw, ldo, pair_offset, stream,   \
                                                                 nullptr, fuse);                                           \
    } while (0)
    if (M <= 8) GM_GO(1, 1);
    if (M <= 16) GM_GO(2, 1);
    if constexpr (!NORM && !ACCUM) {          // the fusions are built for the row counts they are used at
        if (M <= 32) GM_GO(4, 1);
        GM_GO(8, 2);
    }
    return TTB_ERR_UNSUPPORTED;
#undef GM_GO
}

template <bool NORM>
static int gemv_mma_dispatch(const void* x, const void* w, void* out, int out_dtype, int M, int N, int K, int ldx, int ldw,
                             int ldo, int pair_rows, const GmFuse* fuse, cudaStream_t stream) {
    const bool f32 = out_dtype == TTB_DTYPE_F32;
    if (fuse != nullptr && fuse->residual != nullptr) {       // the result goes to the stream: `out` and its type play no part
        if (gemv_mma_half(M, N))
            return gemv_mma_by_rows<GM_HALF, float, NORM, true>(x, w, out, M, N, K, ldx, ldw, ldo, 0, stream, fuse);
        return gemv_mma_by_rows<GM_FULL, float, NORM, true>(x, w, out, M, N, K, ldx, ldw, ldo, 0, stream, fuse);
    }
    if (pair_rows > 0) {
        return f32 ? gemv_mma_by_rows<GM_PAIR, float, NORM>(x, w, out, M, N, K, ldx, ldw, ldo, pair_rows, stream, fuse)
                   : gemv_mma_by_rows<GM_PAIR, __nv_bfloat16, NORM>(x, w, out, M, N, K, ldx, ldw, ldo, pair_rows, stream, fuse);
    }
    if (gemv_mma_half(M, N))
        return f32 ? gemv_mma_by_rows<GM_HALF, float, NORM>(x, w, out, M, N, K, ldx, ldw, ldo, 0, stream, fuse)
                   : gemv_mma_by_rows<GM_HALF, __nv_bfloat16, NORM>(x, w, out, M, N, K, ldx, ldw, ldo, 0, stream, fuse);
    return f32 ? gemv_mma_by_rows<GM_FULL, float, NORM>(x, w, out, M, N, K, ldx, ldw, ldo, 0, stream, fuse)
               : gemv_mma_by_rows<GM_FULL, __nv_bfloat16, NORM>(x, w, out, M, N, K, ldx, ldw, ldo, 0, stream, fuse);
}

// x [M, K] bfloat16, w [N, K] bfloat16, out [M, N] bfloat16 or float32; M <= 64, K a multiple of 8.
// pair_rows > 0: w holds N gate rows followed (pair_rows rows further down) by N up rows, and
// out[m, n] = silu(x . gate_n) * (x . up_n).
TTB_EXPORT int ttb_gemv_mma(const void* x, const void* w, void* out, int out_dtype, int M, int N, int K, int ldx,
                            int ldw, int ldo, int pair_rows, cudaStream_t stream) {
    if (M == 0 || N == 0) return TTB_OK;
    if (!x || !w || !out) return TTB_ERR_ARGUMENT;
    if (M > 64 || K < 8 || (K & 7) || (ldx & 7) || (ldw & 7) || !aligned16(x) || !aligned16(w)) return TTB_ERR_UNSUPPORTED;
    if (out_dtype != TTB_DTYPE_F32 && out_dtype != TTB_DTYPE_BF16) return TTB_ERR_UNSUPPORTED;
    return gemv_mma_dispatch<false>(x, w, out, out_dtype, M, N, K, ldx, ldw, ldo, pair_rows, nullptr, stream);
}

// How many blocks the product of an [M <= 16, K] x with an [N, K] w runs as: the first extent of the
// partial sums of squares that ttb_gemv_mma_fused writes.
TTB_EXPORT int ttb_gemv_mma_parts(int M, int N) {
    const int rows = gemv_mma_half(M, N) ? 8 : 16;
    return (N + rows - 1) / rows;
}

// The same product with the steps around it fused in (M <= 16), see the head of this file.
//   ssq_in != null: x is g * residual (bfloat16) and the results are divided by the rows' RMS, taken from the
//       partial sums ssq_in [ssq_parts][16] and eps;
//   residual != null: the product is added to the float32 matrix residual [M, ldr] and `out` is not written (not
//       with pair_rows); with next_weight [N] float32 also xg [M, ldxg] = bfloat16(next_weight * residual) and
//       ssq_out [ttb_gemv_mma_parts(M, N)][16] are written.
TTB_EXPORT int ttb_gemv_mma_fused(const void* x, const float* ssq_in, int ssq_parts, float eps, const void* w, void* out,
                                  int out_dtype, int M, int N, int K, int ldx, int ldw, int ldo, int pair_rows,
                                  float* residual, int ldr, const float* next_weight, void* xg, int ldxg, float* ssq_out,
                                  cudaStream_t stream) {
    if (M == 0 || N == 0) return TTB_OK;
    if (!x || !w || (!out && !residual)) return TTB_ERR_ARGUMENT;
    if (residual && pair_rows > 0) return TTB_ERR_ARGUMENT;
    if (next_weight && (!residual || !xg || !ssq_out)) return TTB_ERR_ARGUMENT;
    if (ssq_in && ssq_parts < 1) return TTB_ERR_ARGUMENT;
    if (M > 16 || K < 8 || (K & 7) || (ldx & 7) || (ldw & 7) || !aligned16(x) || !aligned16(w)) return TTB_ERR_UNSUPPORTED;
    if (out_dtype != TTB_DTYPE_F32 && out_dtype != TTB_DTYPE_BF16) return TTB_ERR_UNSUPPORTED;
    GmFuse fuse = {ssq_in, ssq_parts, eps, residual, ldr, next_weight, next_weight ? (__nv_bfloat16*)xg : nullptr, ldxg, ssq_out};
    if (ssq_in) return gemv_mma_dispatch<true>(x, w, out, out_dtype, M, N, K, ldx, ldw, ldo, pair_rows, &fuse, stream);
    return gemv_mma_dispatch<false>(x, w, out, out_dtype, M, N, K, ldx, ldw, ldo, pair_rows, &fuse, stream);
}


// The QKV projection of a decode step fused with the rotation and the cache write.
// x [M <= 16, K], w [(heads + 2 kv_heads) * head_dim, K] (queries, keys, values stacked), bfloat16;
// q_out [M, heads * head_dim] gets the rotated queries; rotated keys and the values go to their
// pages. head_dim a multiple of 16, full rotary (every pair of a head is rotated).
// ssq_in != null: x is g * residual and the projection is divided by the rows' RMS (see above).
TTB_EXPORT int ttb_gemv_qkv_rope(const void* x, const float* ssq_in, int ssq_parts, float eps, const void* w, void* q_out,
                                 int M, int K, int ldx, int ldw,
                                 const int* positions, const int* seg_of_token, const float* inv_freq, int heads,
                                 int kv_heads, int head_dim, void* key_pages, void* value_pages,
                                 const int* block_table, int table_width, int page_size, int num_pages, int write_kv,
                                 int* status, cudaStream_t stream) {
    if (M == 0) return TTB_OK;
    if (!x || !w || !q_out || !positions || !inv_freq || !status) return TTB_ERR_ARGUMENT;
    if (write_kv && (!seg_of_token || !key_pages || !value_pages || !block_table)) return TTB_ERR_ARGUMENT;
    if (ssq_in && ssq_parts < 1) return TTB_ERR_ARGUMENT;
    if (M > 16 || K < 8 || (K & 7) || (ldx & 7) || (ldw & 7) || !aligned16(x) || !aligned16(w)) return TTB_ERR_UNSUPPORTED;
    if (head_dim < 16 || (head_dim & 15)) return TTB_ERR_UNSUPPORTED;
    GmRope rope = {positions, seg_of_token, inv_freq, block_table, (__nv_bfloat16*)key_pages, (__nv_bfloat16*)value_pages,
                   status, table_width, page_size, num_pages, heads, kv_heads, head_dim, write_kv};
    GmFuse fuse = {ssq_in, ssq_parts, eps, nullptr, 0, nullptr, nullptr, 0, nullptr};
    const int N = (heads + 2 * kv_heads) * head_dim;
    if (M > 8) {            // two blocks of eight tokens against the same weight fragments
        if (ssq_in)
            return gemv_mma_launch<2, 1, GM_ROPE, 8, __nv_bfloat16, true>(x, w, q_out, M, N, K, ldx, ldw, heads * head_dim,
                                                                          head_dim / 2, stream, &rope, &fuse);
        return gemv_mma_launch<2, 1, GM_ROPE, 8, __nv_bfloat16>(x, w, q_out, M, N, K, ldx, ldw, heads * head_dim,
                                                                head_dim / 2, stream, &rope);
    }
    if (ssq_in)
        return gemv_mma_launch<1, 1, GM_ROPE, 8, __nv_bfloat16, true>(x, w, q_out, M, N, K, ldx, ldw, heads * head_dim,
                                                                      head_dim / 2, stream, &rope, &fuse);
    return gemv_mma_launch<1, 1, GM_ROPE, 8, __nv_bfloat16>(x, w, q_out, M, N, K, ldx, ldw, heads * head_dim,
                                                            head_dim / 2, stream, &rope);
}
