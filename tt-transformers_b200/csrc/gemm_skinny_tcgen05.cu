// C[M, N] = X[M, K] * W[N, K]^T for 9 to 64 rows of X (decode steps of many requests) on the fifth-generation
// tensor cores: the product is bound by streaming W once, so W is the operand that fills the tensor core's M
// side and the few rows of X sit on its N side.
//
// A block owns 128 rows of W (two TMA boxes of 64 rows; with SWIGLU 64 gate rows and their 64 up rows) and a
// slice of K. Per k-block of 64: TMA brings 16 KB of W and NX x 128 bytes of X (NX = 32 or 64 rows, rows
// beyond M read as zero) into a ring of stages; one thread issues four tcgen05.mma (M = 128, N = NX, K = 16)
// that accumulate C^T [128 rows of W, NX rows of X] in tensor memory. The slices of K of one row tile are the
// blocks of one thread-block cluster (1, 2, 4 or 8): each leaves its float32 partial result in its own shared
// memory, and after a cluster barrier the block of rank r sums, in the order of the ranks, the rows of X
// r * NX / S .. through distributed shared memory and stores them (with SWIGLU: silu(gate) * up). So W is
// read once, by as many blocks as fill the GPU, and the result does not depend on the order in which blocks
// finish.
//
// Roles: warp 0 producer (one thread), warp 1 allocates tensor memory and issues the products (one thread),
// warps 2-5 read the accumulator (a warp may only touch lanes 32 * (warp % 4) ..). No load uses cluster
// multicast. Every wait on an mbarrier is bounded: a role that runs out of patience records a code in
// *error_flag and goes on to the block's barriers, so that nobody in the cluster waits for it forever.
// Sizes: M up to 64, any N, K a multiple of 8, row strides of 16 bytes.
//
// ROPE: the fused QKV projection of a decode step with more tokens than the mma.sync skinny kernel takes. W holds
// the query, key and value rows of all heads; a tile of 128 rows holds whole heads (head sizes that divide 128), so
// the rank that finishes a row of X has both halves of every rotation pair (i, i + head_dim / 2) at hand: it rotates
// queries and keys by the token's position (float32 angles, accurate sincosf), writes the queries out and puts keys
// and values straight into their cache pages. No rotation kernel, no round trip of the projection through memory.
#include <cuda.h>

#include "common.cuh"

#define SK_BW 128                     // rows of W per block
#define SK_BK 64
#define SK_THREADS 192
#define SK_MAX_STAGES 4               // two blocks fit an SM: the next kernel moves in while this one drains
#define SK_WAIT_LIMIT (1u << 20)
#define SK_W_BYTES (SK_BW * SK_BK * 2)

#define SK_ERR_PRODUCER 31
#define SK_ERR_MMA 32
#define SK_ERR_EPILOGUE 33

__device__ __forceinline__ uint32_t sk_smem(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void sk_mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void sk_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool sk_wait(uint32_t bar, uint32_t parity) {
    for (uint32_t i = 0; i < SK_WAIT_LIMIT; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.b32 %0, 1, 0, p;\n\t}"
            : "=r"(done) : "r"(bar), "r"(parity) : "memory");
        if (done) return true;
    }
    return false;
}
__device__ __forceinline__ void sk_tma_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(dst), "l"(map), "r"(c0), "r"(c1), "r"(bar) : "memory");
}
__device__ __forceinline__ void sk_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void sk_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void sk_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void sk_mma(uint32_t tmem_c, uint64_t desc_a, uint64_t desc_b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_c), "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate) : "memory");
}
__device__ __forceinline__ void sk_load32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr) : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// K-major tile of rows x 64 bfloat16 in the 128-byte swizzle; groups of eight rows 1,024 bytes apart
__device__ __forceinline__ uint64_t sk_desc(uint32_t addr) {
    uint64_t d = 0;
    d |= (uint64_t)((addr & 0x3FFFF) >> 4);
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}
// four floats of the block of rank `rank` of this cluster, at the address that `local` has in this block
__device__ __forceinline__ float4 sk_ld_cluster4(uint32_t local, uint32_t rank) {
    uint32_t remote;
    float4 v;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(rank));
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(remote) : "memory");
    return v;
}
__device__ __forceinline__ void sk_cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// What the fused QKV form needs beyond the product: positions, rotation frequencies and the cache.
struct SkRope {
    const int* positions;        // [M]
    const int* seg_of_token;     // [M]
    const float* inv_freq;       // [head_dim / 2]
    const int* block_table;      // [segments, table_width]
    __nv_bfloat16* key_pages;    // [num_pages, kv_heads, page_size, head_dim]
    __nv_bfloat16* value_pages;
    int* status;
    int table_width, page_size, num_pages, heads, kv_heads, head_dim, write_kv;
};

#define SK_PLAIN 0
#define SK_SWIGLU 1
#define SK_ROPE 2

struct SkBars {
    uint64_t full[SK_MAX_STAGES], empty[SK_MAX_STAGES], acc_full;
};

// grid (row tiles of W, 1, S), cluster (1, 1, S): blockIdx.z is the block's rank in its cluster and its slice of K.
template <int NX, int MODE, typename TO>
__global__ void __launch_bounds__(SK_THREADS)
gemm_skinny_tcgen05_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                           TO* __restrict__ out, int M, int N, int K, int ldc, int up_offset, int k_per_split,
                           int stages_n, int* __restrict__ error_flag, const SkRope rope) {
    constexpr bool SWIGLU = MODE == SK_SWIGLU;
    constexpr int X_BYTES = NX * SK_BK * 2;
    constexpr int STAGE_BYTES = SK_W_BYTES + X_BYTES;
    extern __shared__ unsigned char sk_raw[];
    unsigned char* stages = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(sk_raw) + 1023) & ~(uintptr_t)1023);
    // the partial result [NX][128] float32 takes the place of the stages once every product has completed
    float* partial = reinterpret_cast<float*>(stages);
    SkBars* bars = reinterpret_cast<SkBars*>(stages + stages_n * STAGE_BYTES);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tile = blockIdx.x, split = blockIdx.z, S = gridDim.z;
    const int out_cols = SWIGLU ? SK_BW / 2 : SK_BW;
    const int n0 = tile * out_cols;                               // first column of C of this tile
    const int row0 = n0, row1 = SWIGLU ? up_offset + n0 : n0 + 64; // first rows of W of the two boxes
    const int k_begin = split * k_per_split;
    const int k_end = min(K, k_begin + k_per_split);
    const int k_blocks = k_begin < k_end ? (k_end - k_begin + SK_BK - 1) / SK_BK : 0;

    if (tid == 0) {
        for (int s = 0; s < stages_n; ++s) {
            sk_mbar_init(sk_smem(&bars->full[s]), 1);
            sk_mbar_init(sk_smem(&bars->empty[s]), 1);
        }
        sk_mbar_init(sk_smem(&bars->acc_full), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(sk_smem(tmem_slot)), "r"((uint32_t)NX) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    sk_fence_before();
    __syncthreads();
    sk_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------------ producer
        if (lane == 0) {
            pdl_wait();                                            // X is the output of the kernel before
            for (int kb = 0; kb < k_blocks; ++kb) {
                const int s = kb % stages_n;
                if (kb >= stages_n && !sk_wait(sk_smem(&bars->empty[s]), ((kb / stages_n) - 1) & 1)) {
                    atomicExch(error_flag, SK_ERR_PRODUCER);
                    break;
                }
                const uint32_t bar = sk_smem(&bars->full[s]);
                const uint32_t dst = sk_smem(stages) + s * STAGE_BYTES;
                const int k = k_begin + kb * SK_BK;
                sk_expect_tx(bar, STAGE_BYTES);                    // whole boxes, whatever lies outside the matrices
                sk_tma_2d(dst, &map_w, k, row0, bar);
                sk_tma_2d(dst + SK_W_BYTES / 2, &map_w, k, row1, bar);
                sk_tma_2d(dst + SK_W_BYTES, &map_x, k, 0, bar);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------------ products
        if (lane == 0) {
            // float32 accumulator, bfloat16 operands, both K-major, M = 128, N = NX
            const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(NX >> 3) << 17) | ((uint32_t)(SK_BW >> 4) << 24);
            bool ok = true;
            for (int kb = 0; kb < k_blocks; ++kb) {
                const int s = kb % stages_n;
                if (!sk_wait(sk_smem(&bars->full[s]), (kb / stages_n) & 1)) {
                    atomicExch(error_flag, SK_ERR_MMA);
                    ok = false;
                    break;
                }
                sk_fence_after();
                const uint32_t wa = sk_smem(stages) + s * STAGE_BYTES, xa = wa + SK_W_BYTES;
#pragma unroll
                for (int k = 0; k < SK_BK / 16; ++k)
                    sk_mma(tmem, sk_desc(wa + k * 32), sk_desc(xa + k * 32), idesc, (kb > 0 || k > 0) ? 1u : 0u);
                sk_commit(sk_smem(&bars->empty[s]));
            }
            if (ok && k_blocks > 0) sk_commit(sk_smem(&bars->acc_full));
        }
    }
    // ---------------------------------------------------------------------- the accumulator comes to shared memory
    if (warp >= 2) {
        // acc_full covers every product of this block, and a product that has completed has read its stage:
        // from here on the stages are free, and the partial result may lie over them
        bool have = k_blocks > 0;
        if (have && !sk_wait(sk_smem(&bars->acc_full), 0)) {
            if (lane == 0) atomicExch(error_flag, SK_ERR_EPILOGUE);
            have = false;
        }
        sk_fence_after();
        const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        const int t = (warp & 3) * 32 + lane;                      // row of W within the tile
#pragma unroll
        for (int c = 0; c < NX; c += 32) {
            uint32_t r[32];
            if (have) {
                sk_load32(lane_base + c, r);
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) r[i] = 0u;
            }
#pragma unroll
            for (int i = 0; i < 32; ++i) partial[(c + i) * SK_BW + t] = __uint_as_float(r[i]);
        }
        sk_fence_before();
    }
    pdl_launch_dependents();
    __syncthreads();
    if (S > 1) sk_cluster_sync();
    // ---------------------------------------------------------------------- rank r finishes its share of the rows of X
    if (MODE == SK_ROPE) {
        // An item is four consecutive elements of the first half of one head of one row of X, and their rotation
        // partners half a head further on: 128 / 8 items a row of X.
        const int rows_per_rank = NX / S;
        const int m_first = split * rows_per_rank, m_last = min(M, m_first + rows_per_rank);
        const int hd = rope.head_dim, half = hd >> 1;
        const int groups = half >> 2;                                 // items per head
        const int per_row = (SK_BW / hd) * groups;                    // = 16
        const int items = m_first < m_last ? (m_last - m_first) * per_row : 0;
        for (int i = tid; i < items; i += SK_THREADS) {
            const int m = m_first + i / per_row, rest = i % per_row;
            const int t = (rest / groups) * hd + (rest % groups) * 4;         // column of the tile: head and pair index
            const float* src = partial + m * SK_BW + t;
            float4 p[8], q[8];
            if (S > 1) {
                const uint32_t a = sk_smem(src);
#pragma unroll
                for (int r = 0; r < 8; ++r)
                    if (r < S) {
                        p[r] = sk_ld_cluster4(a, r);
                        q[r] = sk_ld_cluster4(a + half * 4, r);
                    }
            } else {
                p[0] = *reinterpret_cast<const float4*>(src);
                q[0] = *reinterpret_cast<const float4*>(src + half);
            }
            float lower[4] = {0.f, 0.f, 0.f, 0.f}, upper[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int r = 0; r < 8; ++r)
                if (r < S) {
                    lower[0] += p[r].x; lower[1] += p[r].y; lower[2] += p[r].z; lower[3] += p[r].w;
                    upper[0] += q[r].x; upper[1] += q[r].y; upper[2] += q[r].z; upper[3] += q[r].w;
                }
            const int n = n0 + t;                                    // row of W = element of the QKV row
            if (n >= N) continue;
            const int head = n / hd, e = n - head * hd;              // e < half, a multiple of 4
            const bool is_q = head < rope.heads, is_k = !is_q && head < rope.heads + rope.kv_heads;
            const int pos = rope.positions[m];
            if (is_q || is_k) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float sn, cs;
                    sincosf((float)pos * rope.inv_freq[e + j], &sn, &cs);
                    const float u = lower[j], v = upper[j];
                    lower[j] = u * cs - v * sn;
                    upper[j] = v * cs + u * sn;
                }
            }
            __nv_bfloat162 l01 = __floats2bfloat162_rn(lower[0], lower[1]), l23 = __floats2bfloat162_rn(lower[2], lower[3]);
            __nv_bfloat162 u01 = __floats2bfloat162_rn(upper[0], upper[1]), u23 = __floats2bfloat162_rn(upper[2], upper[3]);
            uint2 lo2, up2;
            lo2.x = *reinterpret_cast<uint32_t*>(&l01); lo2.y = *reinterpret_cast<uint32_t*>(&l23);
            up2.x = *reinterpret_cast<uint32_t*>(&u01); up2.y = *reinterpret_cast<uint32_t*>(&u23);
            __nv_bfloat16* dst = nullptr;
            if (is_q) {
                dst = reinterpret_cast<__nv_bfloat16*>(out) + (size_t)m * ldc + n;
            } else if (rope.write_kv) {
                const int kvh = head - rope.heads - (is_k ? 0 : rope.kv_heads);
                const int page_index = pos / rope.page_size;
                int page = -1;
                if (page_index < rope.table_width)
                    page = rope.block_table[(size_t)rope.seg_of_token[m] * rope.table_width + page_index];
                if ((unsigned)page >= (unsigned)rope.num_pages)
                    atomicExch(rope.status, 0x2000000 + m);          // outside the pool: skip the write, say so
                else
                    dst = (is_k ? rope.key_pages : rope.value_pages) +
                          (((size_t)page * rope.kv_heads + kvh) * rope.page_size + (pos - page_index * rope.page_size)) * hd + e;
            }
            if (dst != nullptr) {
                *reinterpret_cast<uint2*>(dst) = lo2;
                *reinterpret_cast<uint2*>(dst + half) = up2;
            }
        }
    } else {
        // An item is four consecutive columns of one row of X. All of an item's loads from the other blocks are
        // issued before the first sum, so that they are in flight together; the sums run in the order of the ranks.
        const int rows_per_rank = NX / S;
        const int m_first = split * rows_per_rank, m_last = min(M, m_first + rows_per_rank);
        constexpr int GROUPS = (SWIGLU ? SK_BW / 2 : SK_BW) / 4;
        const int items = m_first < m_last ? (m_last - m_first) * GROUPS : 0;
        for (int i = tid; i < items; i += SK_THREADS) {
            const int m = m_first + i / GROUPS, t = (i % GROUPS) * 4;
            const float* src = partial + m * SK_BW + t;
            float4 p[8], q[8];
            if (S > 1) {
                const uint32_t a = sk_smem(src);
#pragma unroll
                for (int r = 0; r < 8; ++r)
                    if (r < S) {
                        p[r] = sk_ld_cluster4(a, r);
                        if (SWIGLU) q[r] = sk_ld_cluster4(a + 64 * 4, r);
                    }
            } else {
                p[0] = *reinterpret_cast<const float4*>(src);
                if (SWIGLU) q[0] = *reinterpret_cast<const float4*>(src + 64);
            }
            float v[4] = {0.f, 0.f, 0.f, 0.f}, u[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int r = 0; r < 8; ++r)
                if (r < S) {
                    v[0] += p[r].x; v[1] += p[r].y; v[2] += p[r].z; v[3] += p[r].w;
                    if (SWIGLU) { u[0] += q[r].x; u[1] += q[r].y; u[2] += q[r].z; u[3] += q[r].w; }
                }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (SWIGLU) v[j] = v[j] * __fdividef(1.f, 1.f + __expf(-v[j])) * u[j];
                if (n0 + t + j < N) out[(size_t)m * ldc + n0 + t + j] = from_float<TO>(v[j]);
            }
        }
    }
    if (S > 1) sk_cluster_sync();    // nobody leaves while its shared memory may still be read
    sk_fence_before();
    __syncthreads();
    if (warp == 1) {
        sk_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)NX) : "memory");
    }
}

// ---------------------------------------------------------------------------- host side
typedef CUresult (*SkEncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                               const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                               CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static SkEncodeFn sk_encode_fn() {
    static SkEncodeFn fn = nullptr;
    static bool looked = false;
    if (!looked) {
        looked = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<SkEncodeFn>(p);
    }
    return fn;
}

// A row-major [rows, cols] bfloat16 matrix with row stride ld (elements), fetched in boxes of box_rows x 64.
static bool sk_make_map(CUtensorMap* map, const void* base, int rows, int cols, int ld, int box_rows) {
    SkEncodeFn encode = sk_encode_fn();
    if (!encode) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {SK_BK, (cuuint32_t)box_rows};
    cuuint32_t elem[2] = {1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int sk_sm_count() {
    static int count = 0;
    if (count == 0) {
        int device = 0;
        cudaGetDevice(&device);
        cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device);
        if (count <= 0) count = 1;
    }
    return count;
}

// Slices of K (= blocks of a cluster) for a product with this many row tiles of W: as many, of 1, 2, 4 and 8, as
// keep the grid within two blocks an SM and leave every slice at least four k-blocks. TTB200_SKINNY_SPLITS forces it.
static int sk_splits(int tiles, int K) {
    static int forced = -1;
    if (forced < 0) {
        const char* e = getenv("TTB200_SKINNY_SPLITS");
        forced = e ? atoi(e) : 0;
    }
    if (forced == 1 || forced == 2 || forced == 4 || forced == 8) return forced;
    const int k_blocks = (K + SK_BK - 1) / SK_BK;
    int s = 1;
    while (s < 8 && tiles * (2 * s) <= 2 * sk_sm_count() && k_blocks / (2 * s) >= 4) s *= 2;
    return s;
}

template <int NX, int MODE, typename TO>
static int sk_launch(const CUtensorMap& map_w, const CUtensorMap& map_x, void* C, int M, int N, int K, int ldc,
                     int up_offset, int* error_flag, cudaStream_t stream, const SkRope* rope = nullptr) {
    constexpr bool SWIGLU = MODE == SK_SWIGLU;
    auto kernel = gemm_skinny_tcgen05_kernel<NX, MODE, TO>;
    const size_t stage_bytes = SK_W_BYTES + NX * SK_BK * 2;
    static TtbOncePerDevice configured;
    if (configured.pending()) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)(1024 + SK_MAX_STAGES * stage_bytes + sizeof(SkBars) + 16));
        if (e != cudaSuccess) return (int)e;
        configured.mark();
    }
    const int out_cols = SWIGLU ? SK_BW / 2 : SK_BW;
    const int tiles = (N + out_cols - 1) / out_cols;
    const int S = sk_splits(tiles, K);
    // (eight stages and one block an SM for grids that fit the GPU once were measured: twice as slow back to
    // back, since the blocks of the next launch cannot become resident beside them)
    const int stages_n = SK_MAX_STAGES;
    const size_t smem = 1024 + stages_n * stage_bytes + sizeof(SkBars) + 16;
    const int k_blocks = (K + SK_BK - 1) / SK_BK;
    const int k_per_split = (k_blocks + S - 1) / S * SK_BK;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(tiles, 1, S);
    cfg.blockDim = dim3(SK_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    int n_attr = 0;
    if (ttb_pdl_enabled()) {
        attr[n_attr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n_attr].val.programmaticStreamSerializationAllowed = 1;
        ++n_attr;
    }
    if (S > 1) {
        attr[n_attr].id = cudaLaunchAttributeClusterDimension;
        attr[n_attr].val.clusterDim.x = 1;
        attr[n_attr].val.clusterDim.y = 1;
        attr[n_attr].val.clusterDim.z = S;
        ++n_attr;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n_attr;
    const SkRope none = {};
    cudaLaunchKernelEx(&cfg, kernel, map_w, map_x, (TO*)C, M, N, K, ldc, up_offset, k_per_split, stages_n, error_flag,
                       rope ? *rope : none);
    return ttb_launch_status();
}

TTB_EXPORT int ttb_gemm_skinny_tcgen05_rows() { return 64; }

// X [M, K] with M <= 64, W [N, K] (or [2 * swiglu_rows, K] with swiglu_rows = N gate rows then N up rows), bfloat16,
// K-contiguous. C [M, N] bfloat16 or float32. error_flag: device int that a timed-out wait sets (0 = fine).
TTB_EXPORT int ttb_gemm_skinny_tcgen05(const void* X, const void* W, void* C, int out_dtype, int M, int N, int K, int ldx,
                                       int ldw, int ldc, int swiglu_rows, int* error_flag, cudaStream_t stream) {
    if (M == 0 || N == 0) return TTB_OK;
    if (!X || !W || !C || !error_flag) return TTB_ERR_ARGUMENT;
    if (M > 64 || K < 8 || (K & 7) || (ldx & 7) || (ldw & 7) || !aligned16(X) || !aligned16(W)) return TTB_ERR_UNSUPPORTED;
    if (swiglu_rows != 0 && swiglu_rows != N) return TTB_ERR_ARGUMENT;
    const bool f32 = out_dtype == TTB_DTYPE_F32;
    if (!f32 && out_dtype != TTB_DTYPE_BF16) return TTB_ERR_UNSUPPORTED;
    const int nx = M <= 32 ? 32 : 64;
    CUtensorMap map_w, map_x;
    if (!sk_make_map(&map_w, W, swiglu_rows ? 2 * N : N, K, ldw, 64)) return TTB_ERR_UNSUPPORTED;
    if (!sk_make_map(&map_x, X, M, K, ldx, nx)) return TTB_ERR_UNSUPPORTED;
#define SK_ARGS map_w, map_x, C, M, N, K, ldc, swiglu_rows, error_flag, stream
    if (nx == 32) {
        if (swiglu_rows) return f32 ? sk_launch<32, SK_SWIGLU, float>(SK_ARGS) : sk_launch<32, SK_SWIGLU, __nv_bfloat16>(SK_ARGS);
        return f32 ? sk_launch<32, SK_PLAIN, float>(SK_ARGS) : sk_launch<32, SK_PLAIN, __nv_bfloat16>(SK_ARGS);
    }
    if (swiglu_rows) return f32 ? sk_launch<64, SK_SWIGLU, float>(SK_ARGS) : sk_launch<64, SK_SWIGLU, __nv_bfloat16>(SK_ARGS);
    return f32 ? sk_launch<64, SK_PLAIN, float>(SK_ARGS) : sk_launch<64, SK_PLAIN, __nv_bfloat16>(SK_ARGS);
#undef SK_ARGS
}

// The QKV projection of a decode step fused with the rotation and the cache write, for up to 64 tokens.
// X [M, K], W [(heads + 2 kv_heads) * head_dim, K] (queries, keys, values stacked), bfloat16; q_out [M, heads *
// head_dim] gets the rotated queries; rotated keys and the values go to their pages [num_pages, kv_heads,
// page_size, head_dim]. head_dim 16, 32, 64 or 128 (whole heads in a tile of 128 rows), full rotary (every pair
// (i, i + head_dim / 2) of a head is rotated).
TTB_EXPORT int ttb_gemm_skinny_tcgen05_qkv_rope(const void* X, const void* W, void* q_out, int M, int K, int ldx, int ldw,
                                                const int* positions, const int* seg_of_token, const float* inv_freq,
                                                int heads, int kv_heads, int head_dim, void* key_pages, void* value_pages,
                                                const int* block_table, int table_width, int page_size, int num_pages,
                                                int write_kv, int* status, int* error_flag, cudaStream_t stream) {
    if (M == 0) return TTB_OK;
    if (!X || !W || !q_out || !positions || !inv_freq || !status || !error_flag) return TTB_ERR_ARGUMENT;
    if (write_kv && (!seg_of_token || !key_pages || !value_pages || !block_table)) return TTB_ERR_ARGUMENT;
    if (M > 64 || K < 8 || (K & 7) || (ldx & 7) || (ldw & 7) || !aligned16(X) || !aligned16(W)) return TTB_ERR_UNSUPPORTED;
    if (head_dim != 16 && head_dim != 32 && head_dim != 64 && head_dim != 128) return TTB_ERR_UNSUPPORTED;
    if (heads < 1 || kv_heads < 1 || (reinterpret_cast<uintptr_t>(q_out) & 7u) || (reinterpret_cast<uintptr_t>(key_pages) & 7u) ||
        (reinterpret_cast<uintptr_t>(value_pages) & 7u))
        return TTB_ERR_UNSUPPORTED;
    const int N = (heads + 2 * kv_heads) * head_dim;
    const int nx = M <= 32 ? 32 : 64;
    CUtensorMap map_w, map_x;
    if (!sk_make_map(&map_w, W, N, K, ldw, 64)) return TTB_ERR_UNSUPPORTED;
    if (!sk_make_map(&map_x, X, M, K, ldx, nx)) return TTB_ERR_UNSUPPORTED;
    SkRope rope = {positions, seg_of_token, inv_freq, block_table, (__nv_bfloat16*)key_pages, (__nv_bfloat16*)value_pages,
                   status, table_width, page_size, num_pages, heads, kv_heads, head_dim, write_kv};
    if (nx == 32)
        return sk_launch<32, SK_ROPE, __nv_bfloat16>(map_w, map_x, q_out, M, N, K, heads * head_dim, 0, error_flag, stream, &rope);
    return sk_launch<64, SK_ROPE, __nv_bfloat16>(map_w, map_x, q_out, M, N, K, heads * head_dim, 0, error_flag, stream, &rope);
}
