// Weight-streaming product for a handful of decoded tokens (M <= 8) as a persistent kernel:
//   out[m, n] = sum_k x[m, k] * w[n, k],   or with `pair_rows`: silu(x . gate_n) * (x . up_n).
// One block of 16 warps per SM; the rows of w are dealt out evenly over the blocks (a block gets 13 or 14 of
// 2,048 rows, 55 or 56 of 8,192 row pairs on 148 SMs), and the weights a block needs form ONE stream that every
// thread fetches with 16-byte cp.async copies into a ring of its own in shared memory, GR_DEPTH steps ahead of
// use. The stream runs on across the block's row tiles, and it starts before the wait for the kernel in front
// (weights depend on no kernel), so memory is busy from the block's first cycle to its last but one. The
// mma.sync skinny kernel (gemv_mma.cu) runs the same product as hundreds of short blocks that each load, add up
// and leave, and every one of them reads x again. Which of the two a product goes to was settled by timing whole
// decode steps (kernels/__init__.py, `ring_gemv`): this one for the output projection at 1 to 8 rows and for
// gate/up with SwiGLU at 6 to 8.
//
// The product itself is as there: mma.m16n8k16 with the weights as the 16-row operand and the tokens as the
// 8-column one; within a block of 32 k, lane t of a quad holds k = 8t .. 8t+7 of both operands, a permutation of
// k that the sum does not see, so that fragments are plain 16-byte words. The 16 warps share a tile's rows and
// take the k-blocks in turn; their partial sums meet in shared memory, where one warp (another for every tile)
// adds them in the order of the warps and writes the result. x lies in shared memory when it fits beside the
// ring (rows 16 words apart modulo the 32 banks), else its fragments come from L2 four steps ahead.
#include "common.cuh"

#define GR_WARPS 16
#define GR_THREADS (GR_WARPS * 32)
#define GR_DEPTH 4                     // steps of weights in flight per thread (32 bytes each): 64 KB a block
#define GR_RING_BYTES (GR_DEPTH * 2 * GR_THREADS * 16)
#define GR_XAHEAD 4
#define GR_X_SMEM_LIMIT (48 * 1024)    // x goes to shared memory up to this size

struct GrArgs {
    const __nv_bfloat16* x; int ldx;           // [M, K]
    const __nv_bfloat16* w; int ldw;           // [N, K], or [pair_offset + N, K] with pair_offset > 0
    void* out; int ldo;                        // [M, N]
    int M, N, K;
    int pair_offset;                           // > 0: row n pairs with row n + pair_offset (gate and up), SwiGLU epilogue
    int x_stride;                              // elements between the rows of x in shared memory (0: x stays in global memory)
};

// Where this thread's weight loads have got to: the tile, and within it the next step's addresses.
struct GrProducer {
    int tile, left;                  // steps left in this tile; tile == tiles: the stream has ended
    const __nv_bfloat16* pa;         // the next 16 bytes of this lane's first and second row
    const __nv_bfloat16* pb;
    int step_a, step_b;              // elements from step to step: 512 where the row exists, else 0 (and 0 bytes are read)
    int k;                           // this lane's k at the next step
};

__device__ __forceinline__ void gr_cp_async16(uint32_t dst, const void* src, int bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void gr_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N> __device__ __forceinline__ void gr_wait_group() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }
__device__ __forceinline__ void gr_mma(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <bool PAIR, typename TO, bool XSMEM>
__global__ void __launch_bounds__(GR_THREADS, 1) gemv_ring_kernel(const GrArgs a) {
    extern __shared__ __align__(16) unsigned char gr_smem[];
    unsigned char* ring = gr_smem;                                                          // [GR_DEPTH][2][GR_THREADS] x 16 bytes
    float4* partial = reinterpret_cast<float4*>(gr_smem + GR_RING_BYTES);                   // [2][GR_WARPS][32]
    __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(partial + 2 * GR_WARPS * 32);      // [8][x_stride]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
    constexpr int R = PAIR ? 8 : 16;                                                        // rows (row pairs) of a tile
    const int lo = (int)((long long)a.N * blockIdx.x / gridDim.x);
    const int hi = (int)((long long)a.N * (blockIdx.x + 1) / gridDim.x);
    const int tiles = (hi - lo + R - 1) / R;
    const int steps = (a.K + GR_WARPS * 32 - 1) / (GR_WARPS * 32);
    const int K = a.K;
    const int kmine = warp * 32 + t * 8;

    GrProducer p = {};
    auto enter_tile = [&]() {
        const int ra = lo + p.tile * R + g;
        const int rb = PAIR ? ra + a.pair_offset : ra + 8;
        const bool va = ra < hi, vb = PAIR ? va : rb < hi;
        p.k = kmine;
        p.pa = va ? a.w + (size_t)ra * a.ldw + kmine : a.w;
        p.pb = vb ? a.w + (size_t)rb * a.ldw + kmine : a.w;
        p.step_a = va ? GR_WARPS * 32 : 0;
        p.step_b = vb ? GR_WARPS * 32 : 0;
        p.left = steps;
    };
    // the next step of the stream goes into the ring slot at `dst` (nothing, once the stream has ended; a group is
    // committed all the same, so that the count of groups in flight stays GR_DEPTH)
    auto issue = [&](uint32_t dst) {
        if (p.tile < tiles) {
            const bool kin = p.k < K;
            gr_cp_async16(dst, kin ? p.pa : a.w, (kin && p.step_a) ? 16 : 0);      // 0 bytes: zeros, nothing is read
            gr_cp_async16(dst + GR_THREADS * 16, kin ? p.pb : a.w, (kin && p.step_b) ? 16 : 0);
            p.pa += p.step_a;
            p.pb += p.step_b;
            p.k += GR_WARPS * 32;
            if (--p.left == 0 && ++p.tile < tiles) enter_tile();
        }
        gr_commit();
    };
    p.tile = 0;
    if (tiles > 0) enter_tile();
    const uint32_t ring_addr = (uint32_t)__cvta_generic_to_shared(ring + threadIdx.x * 16);
    const unsigned char* ring_mine = ring + threadIdx.x * 16;
#pragma unroll 1
    for (int s = 0; s < GR_DEPTH; ++s) issue(ring_addr + s * (2 * GR_THREADS * 16));
    pdl_wait();                                                   // x is the output of the kernel before

    const uint4 zero = make_uint4(0, 0, 0, 0);
    if (XSMEM) {
        const int chunks = K >> 3;
        for (int i = threadIdx.x; i < 8 * chunks; i += GR_THREADS) {
            const int m = i / chunks, c = (i - m * chunks) * 8;
            *reinterpret_cast<uint4*>(xs + (size_t)m * a.x_stride + c) =
                m < a.M ? *reinterpret_cast<const uint4*>(a.x + (size_t)m * a.ldx + c) : zero;
        }
        __syncthreads();
    }
    const __nv_bfloat16* xmine = XSMEM ? xs + (size_t)g * a.x_stride + kmine : a.x + (size_t)g * a.ldx + kmine;
    const bool xrow = XSMEM || g < a.M;
    auto xload = [&](int it) -> uint4 {
        const int off = it * (GR_WARPS * 32);
        if (!xrow || off + kmine >= K) return zero;
        return *reinterpret_cast<const uint4*>(xmine + off);
    };
    const int total = tiles * steps;
    uint4 xq[GR_XAHEAD];
    int it_ahead = 0;                                             // the `it` of the step GR_XAHEAD after the current one
    if (!XSMEM) {
#pragma unroll
        for (int j = 0; j < GR_XAHEAD; ++j) {
            xq[j] = j < total ? xload(it_ahead) : zero;
            if (++it_ahead == steps) it_ahead = 0;
        }
    }
    TO* out = reinterpret_cast<TO*>(a.out);
    const int m0 = 2 * t, m1 = m0 + 1;
    uint32_t slot_off = 0;
    int parity = 0, q = 0;
#pragma unroll 1
    for (int tile = 0; tile < tiles; ++tile) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
        for (int it = 0; it < steps; ++it, ++q) {
            uint4 xv;
            if (XSMEM) {
                xv = xload(it);
            } else {
                xv = xq[0];
#pragma unroll
                for (int j = 0; j + 1 < GR_XAHEAD; ++j) xq[j] = xq[j + 1];
                xq[GR_XAHEAD - 1] = (q + GR_XAHEAD < total) ? xload(it_ahead) : zero;
                if (++it_ahead == steps) it_ahead = 0;
            }
            gr_wait_group<GR_DEPTH - 1>();
            const uint4 wa = *reinterpret_cast<const uint4*>(ring_mine + slot_off);
            const uint4 wb = *reinterpret_cast<const uint4*>(ring_mine + slot_off + GR_THREADS * 16);
            gr_mma(acc, wa.x, wb.x, wa.y, wb.y, xv.x, xv.y);
            gr_mma(acc, wa.z, wb.z, wa.w, wb.w, xv.z, xv.w);
            issue(ring_addr + slot_off);
            slot_off += 2 * GR_THREADS * 16;
            if (slot_off == GR_RING_BYTES) slot_off = 0;
        }
        if (tile == tiles - 1) pdl_launch_dependents();           // this block's weights have all arrived
        float4* mine = partial + parity * (GR_WARPS * 32);
        mine[warp * 32 + lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        __syncthreads();
        if (warp == (tile & (GR_WARPS - 1))) {                    // this warp adds the tile up and writes it
            float4 s = mine[lane];
#pragma unroll
            for (int w = 1; w < GR_WARPS; ++w) {
                const float4 v = mine[w * 32 + lane];
                s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
            }
            const int row = lo + tile * R + g;
            if (PAIR) {
                if (row < hi) {
                    if (m0 < a.M) out[(size_t)m0 * a.ldo + row] = from_float<TO>(s.x / (1.f + __expf(-s.x)) * s.z);
                    if (m1 < a.M) out[(size_t)m1 * a.ldo + row] = from_float<TO>(s.y / (1.f + __expf(-s.y)) * s.w);
                }
            } else {
                if (row < hi) {
                    if (m0 < a.M) out[(size_t)m0 * a.ldo + row] = from_float<TO>(s.x);
                    if (m1 < a.M) out[(size_t)m1 * a.ldo + row] = from_float<TO>(s.y);
                }
                if (row + 8 < hi) {
                    if (m0 < a.M) out[(size_t)m0 * a.ldo + row + 8] = from_float<TO>(s.z);
                    if (m1 < a.M) out[(size_t)m1 * a.ldo + row + 8] = from_float<TO>(s.w);
                }
            }
        }
        parity ^= 1;
    }
    if (tiles == 0) pdl_launch_dependents();
    gr_wait_group<0>();
}

// Elements between the rows of x in shared memory: rows 16 words apart modulo 32 banks, so that a quarter warp's
// 16-byte reads (two rows, four k-offsets each) fall on different banks.
static int gemv_ring_x_stride(int K) {
    const int words = K / 2;
    const int pad_words = ((16 - words % 32) % 32 + 32) % 32;
    return K + 2 * pad_words;
}

static int gemv_ring_blocks() {
    static int sms[TTB_MAX_DEVICES] = {};
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= TTB_MAX_DEVICES) return 0;
    if (sms[d] == 0) cudaDeviceGetAttribute(&sms[d], cudaDevAttrMultiProcessorCount, d);
    return sms[d];
}

template <bool PAIR, typename TO, bool XSMEM>
static int gemv_ring_launch(const GrArgs& a, size_t smem, cudaStream_t stream) {
    auto kernel = gemv_ring_kernel<PAIR, TO, XSMEM>;
    static TtbOncePerDevice configured;
    if (configured.pending()) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)(GR_RING_BYTES + 2 * GR_WARPS * 32 * sizeof(float4) + GR_X_SMEM_LIMIT + 1024));
        if (e != cudaSuccess) return (int)e;
        configured.mark();
    }
    ttb_launch(kernel, dim3(gemv_ring_blocks()), dim3(GR_THREADS), smem, stream, a);
    return ttb_launch_status();
}

// x [M <= 8, K] bfloat16, w [N, K] bfloat16, out [M, N] bfloat16 or float32; K a multiple of 8, rows 16-byte aligned.
// pair_rows > 0: w holds N gate rows followed (pair_rows rows further down) by N up rows, and
// out[m, n] = silu(x . gate_n) * (x . up_n).
TTB_EXPORT int ttb_gemv_ring(const void* x, const void* w, void* out, int out_dtype, int M, int N, int K, int ldx,
                             int ldw, int ldo, int pair_rows, cudaStream_t stream) {
    if (M == 0 || N == 0) return TTB_OK;
    if (!x || !w || !out) return TTB_ERR_ARGUMENT;
    if (M > 8 || K < 8 || (K & 7) || (ldx & 7) || (ldw & 7) || !aligned16(x) || !aligned16(w)) return TTB_ERR_UNSUPPORTED;
    if (out_dtype != TTB_DTYPE_F32 && out_dtype != TTB_DTYPE_BF16) return TTB_ERR_UNSUPPORTED;
    if (gemv_ring_blocks() < 1) return TTB_ERR_UNSUPPORTED;
    GrArgs a;
    a.x = (const __nv_bfloat16*)x; a.ldx = ldx;
    a.w = (const __nv_bfloat16*)w; a.ldw = ldw;
    a.out = out; a.ldo = ldo;
    a.M = M; a.N = N; a.K = K;
    a.pair_offset = pair_rows;
    const int stride = gemv_ring_x_stride(K);
    const bool xsmem = (size_t)8 * stride * 2 <= GR_X_SMEM_LIMIT;
    a.x_stride = xsmem ? stride : 0;
    const size_t smem = GR_RING_BYTES + 2 * GR_WARPS * 32 * sizeof(float4) + (xsmem ? (size_t)8 * stride * 2 : 0);
    const bool f32 = out_dtype == TTB_DTYPE_F32;
#define GR_GO(PAIR, XS)                                                                                   \
    return f32 ? gemv_ring_launch<PAIR, float, XS>(a, smem, stream) : gemv_ring_launch<PAIR, __nv_bfloat16, XS>(a, smem, stream)
    if (pair_rows > 0) {
        if (xsmem) GR_GO(true, true);
        GR_GO(true, false);
    }
    if (xsmem) GR_GO(false, true);
    GR_GO(false, false);
#undef GR_GO
}
