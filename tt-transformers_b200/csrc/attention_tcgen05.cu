// Paged causal flash attention for prompt portions on the fifth-generation tensor cores, head sizes 64 and 128.
//
// A block owns 128 query rows: 128 / (heads per KV head) tokens of one segment times the query heads of
// one KV head, token-major, so all rows share the keys and values that are loaded. Per tile of 64 keys:
//   producer (warp 0, a lane per copy)  TMA loads of whole cache pages (cp.async.bulk.tensor, 128-byte swizzle,
//                                   no multicast) into a ring of K and V stages; the page ids of the
//                                   block's key range are first copied from the block table to shared memory
//   first product (warp 1, one thread)   S = Q K^T by tcgen05.mma into one of two S buffers in tensor memory, as
//                                   soon as the keys have arrived and the buffer is free: the next tile's S
//                                   is computed under this tile's softmax
//   second product (warp 6, one thread)  once the softmax warps have written P, O += P V into the O accumulator
//                                   in tensor memory, with P as the first operand from tensor memory
//   softmax (warps 2-5)             thread r owns query row r: reads its 64 scores with tcgen05.ld, masks the
//                                   tiles that the causal edge or the end of the key range cuts, keeps the
//                                   running maximum and sum in float32 (no shuffles: a row is one thread),
//                                   rescales its O row in tensor memory when the maximum moved, writes P as
//                                   bfloat16 to tensor memory with tcgen05.st; at the end normalises O
//                                   and stores it (or, with key splits, the unnormalised partial result)
// Every wait on an mbarrier is bounded; a role that runs out of patience sets *error_flag, and the block
// frees its tensor memory and returns. Rows of V beyond the last visible key are zeroed in shared memory
// before they meet a probability of zero, so stale or poisoned cache contents never reach the output.
//
// A head of 128 is two halves of 64 columns everywhere (the 128-byte swizzle's width): Q, K and V tiles are
// [half][rows][64], Q K^T runs over both halves' k-steps, P V is issued once per half of V into its half of O.
// Takes: head sizes 64 and 128; up to 16 heads per KV head; page sizes that are powers of two from 8 on; no window.
// Everything else goes to attention_mma.cu or attention_generic.cu.
#include <cuda.h>

#include "common.cuh"

#define FA_BM 128
#define FA_BN 64
#define FA_MAX_STAGES 3
#define FA_THREADS 224
#define FA_WAIT_LIMIT (1u << 20)
#define FA_TABLE 1024                 // block-table entries kept in shared memory per block
#define FA_TMEM_COLS 256              // S0: 0-63, S1: 64-127 (P over the first 32 columns of each), O: 128 .. 128 + head size
#define FA_P_COL 192                  // first column of separate P buffers (head size 64 with P_ALIAS false: P0 192-223, P1 224-255)

#define FA_HALF_TILE (FA_BN * 128)            // 64 keys x 64 columns of K or V: 8 KB
#define FA_ROWS_TILE (FA_BM * 128)            // 128 rows x 64 columns of Q: 16 KB

__device__ __forceinline__ uint32_t fa_smem(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void fa_mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void fa_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void fa_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool fa_wait(uint32_t bar, uint32_t parity) {
    for (uint32_t i = 0; i < FA_WAIT_LIMIT; ++i) {
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
__device__ __forceinline__ void fa_tma_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(dst), "l"(map), "r"(c0), "r"(c1), "r"(bar) : "memory");
}
__device__ __forceinline__ void fa_tma_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, uint32_t bar) {
    asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
                 ::"r"(dst), "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(bar) : "memory");
}
__device__ __forceinline__ void fa_tma_4d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3, uint32_t bar) {
    asm volatile("cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];"
                 ::"r"(dst), "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar) : "memory");
}
__device__ __forceinline__ void fa_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fa_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fa_fence_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void fa_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void fa_mma(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate) : "memory");
}
// the first operand in tensor memory: row r in lane r, two bfloat16 of the reduction dimension a column
__device__ __forceinline__ void fa_mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t desc_b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(tmem_d), "r"(tmem_a), "l"(desc_b), "r"(idesc), "r"(accumulate) : "memory");
}
__device__ __forceinline__ void fa_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr) : "memory");
}
__device__ __forceinline__ void fa_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
        ::"r"(taddr),
          "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
          "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
          "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void fa_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void fa_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ float fa_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Operand descriptor of a tile with 128-byte rows in the 128-byte swizzle; groups of eight rows are 1,024
// bytes apart. For a K-major operand (Q, K, P) a row is a row of the operand and a k-step of 16 advances
// the start by 32 bytes; for the MN-major operand (V: rows are keys, the reduction dimension) a k-step of
// 16 keys advances the start by 16 rows.
__device__ __forceinline__ uint64_t fa_desc(uint32_t addr) {
    uint64_t d = 0;
    d |= (uint64_t)((addr & 0x3FFFF) >> 4);
    d |= (uint64_t)1 << 16;                          // leading-dimension offset: one atom wide, not used
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

struct FaBars {
    // p_full[b]: the softmax warps have written P buffer b; p_free[b]: the P V that read buffer b has completed
    // (so the buffer, or the S buffer it lies in, may be written again, and O holds that product)
    uint64_t q_full, kv_full[FA_MAX_STAGES], kv_empty[FA_MAX_STAGES], s_full[2], s_empty[2], p_full[2], p_free[2];
};

template <int HD>
__global__ void __launch_bounds__(FA_THREADS, 2)
attention_tcgen05_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                         const __grid_constant__ CUtensorMap map_v, __nv_bfloat16* __restrict__ out,
                         const int* __restrict__ cu_seqlens, const int* __restrict__ seg_pos0,
                         const int* __restrict__ block_table, int table_width, int page_size, int page_shift,
                         const int* __restrict__ qtile_seg, const int* __restrict__ qtile_tok0, int heads, int kv_heads,
                         float scale_log2, int num_splits, float* __restrict__ partial_o,
                         float* __restrict__ partial_ml, int num_pages, int* __restrict__ status,
                         int* __restrict__ error_flag) {
    extern __shared__ __align__(1024) unsigned char fa_raw[];
    unsigned char* base = fa_raw;        // the 128-byte swizzle wants tiles on 1,024-byte boundaries
    constexpr int HALVES = HD / 64;
    // P lives in tensor memory (two buffers of 32 columns, two bfloat16 a column) and is the P V product's
    // first operand from there: no copy through shared memory, no proxy fence. P of tile j overwrites the first
    // 32 columns of the S buffer that its scores came from (a thread has its row of scores in registers by
    // then), and that S buffer is free for tile j + 2 only once the P V of tile j has completed. Head size 128
    // has no other place for P; head size 64 has 64 columns to spare (P_ALIAS false puts P there and hands the
    // S buffer back as soon as it has been read), which measured 1 % slower.
    constexpr int NP = 2;
    constexpr bool P_ALIAS = true;
    constexpr int FA_STAGES = HD == 64 ? 3 : 2;
    constexpr int FA_TILE_BYTES = HALVES * FA_HALF_TILE;        // one K or V stage
    unsigned char* q_tile = base;                               // [half][128 rows][64]
    unsigned char* k_stage = base + HALVES * FA_ROWS_TILE;      // [stage][half][64 keys][64]
    unsigned char* v_stage = k_stage + FA_STAGES * FA_TILE_BYTES;
    FaBars* bars = reinterpret_cast<FaBars*>(v_stage + FA_STAGES * FA_TILE_BYTES);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 1);
    int* page_cache = reinterpret_cast<int*>(tmem_slot + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // The tile list comes sorted, most keys first. Blocks are handed out in the order of their linear index:
    // all KV heads of the longest tile go first, so that the longest blocks do not end the grid.
    const int linear = blockIdx.x + gridDim.x * blockIdx.y, split = blockIdx.z;
    const int qt = linear / kv_heads, g = linear % kv_heads;
    const int rep = heads / kv_heads;
    const int seg = qtile_seg[qt], tok0 = qtile_tok0[qt];
    const int seg_start = cu_seqlens[seg];
    const int seg_tokens = cu_seqlens[seg + 1] - seg_start;
    const int pos0 = seg_pos0[seg];
    const int tokens_per_tile = FA_BM / rep;
    const int tile_tokens = min(tokens_per_tile, seg_tokens - tok0);
    const int valid_rows = tile_tokens * rep;
    const int q_first = pos0 + tok0, q_last = q_first + tile_tokens - 1;
    const int total = q_last + 1;
    const int chunk = ((total + num_splits - 1) / num_splits + FA_BN - 1) / FA_BN * FA_BN;
    const int k_begin = split * chunk;
    const int k_end = min(q_last + 1, k_begin + chunk);
    const int num_tiles = k_begin < k_end ? (k_end - k_begin + FA_BN - 1) / FA_BN : 0;
    const int* table = block_table + (size_t)seg * table_width;
    const int page_base = k_begin >> page_shift;

    if (fa_smem(base) & 1023u) {          // the launch did not honour the alignment asked for above: say so, do nothing
        if (threadIdx.x == 0) atomicExch(error_flag, 17);
        return;
    }
    if (threadIdx.x == 0) {
        fa_mbar_init(fa_smem(&bars->q_full), 1);
        for (int s = 0; s < FA_STAGES; ++s) {
            fa_mbar_init(fa_smem(&bars->kv_full[s]), 1);
            fa_mbar_init(fa_smem(&bars->kv_empty[s]), 1);
        }
        for (int b = 0; b < 2; ++b) {
            fa_mbar_init(fa_smem(&bars->s_full[b]), 1);
            fa_mbar_init(fa_smem(&bars->s_empty[b]), 4);      // one arrival per softmax warp
        }
        for (int b = 0; b < 2; ++b) {
            fa_mbar_init(fa_smem(&bars->p_full[b]), 4);
            fa_mbar_init(fa_smem(&bars->p_free[b]), 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fa_fence_async();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(fa_smem(tmem_slot)), "r"((uint32_t)FA_TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    pdl_wait();                                   // queries and cache pages come from the kernels before
    if (num_tiles > 0) {
        const int last_page = (k_end - 1) >> page_shift;
        const int count = min(last_page - page_base + 1, FA_TABLE);
        for (int i = threadIdx.x; i < count; i += FA_THREADS) {
            int page = table[page_base + i];
            if ((unsigned)page >= (unsigned)num_pages) {          // outside the pool: flag it, read the scratch page
                if (status != nullptr) atomicExch(status, 0x2000000 + seg);
                page = 0;
            }
            page_cache[i] = page;
        }
    }
    fa_fence_before();
    __syncthreads();
    fa_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const uint32_t tmem_o = tmem_base + 2 * FA_BN;

    if (warp == 0) {
        // ------------------------------------------------------------------ producer: one copy per lane
        if (num_tiles > 0) {
            if (lane == 0) {
                fa_expect_tx(fa_smem(&bars->q_full), (uint32_t)(HALVES * rep * tokens_per_tile * 128));      // whole boxes, whatever lies outside
                for (int h = 0; h < HALVES; ++h)
                    fa_tma_4d(fa_smem(q_tile) + h * FA_ROWS_TILE, &map_q, 0, h, g * rep, seg_start + tok0, fa_smem(&bars->q_full));
            }
            const int box_rows = min(page_size, FA_BN);            // a copy brings a page, or 64 rows of a larger one
            const int boxes_per_tile = FA_BN / box_rows;
            for (int j = 0; j < num_tiles; ++j) {
                const int s = j % FA_STAGES;
                if (j >= FA_STAGES) {
                    bool freed = true;
                    if (lane == 0) freed = fa_wait(fa_smem(&bars->kv_empty[s]), ((j / FA_STAGES) - 1) & 1);
                    freed = __shfl_sync(0xffffffffu, freed, 0);
                    if (!freed) {
                        if (lane == 0) atomicExch(error_flag, 11);
                        break;
                    }
                }
                const int key0 = k_begin + j * FA_BN;
                const int boxes = min(boxes_per_tile, ((k_end - key0) + box_rows - 1) / box_rows);
                const uint32_t bar = fa_smem(&bars->kv_full[s]);
                if (lane == 0) fa_expect_tx(bar, (uint32_t)boxes * box_rows * HD * 2 * 2);
                __syncwarp();
                // a lane brings one box: keys or values, one half of the head, one page (or 64 rows of a larger one)
                for (int c = lane; c < 2 * HALVES * boxes; c += 32) {
                    const int which = c & 1, h = (c >> 1) % HALVES, pg = (c >> 1) / HALVES;
                    const int key = key0 + pg * box_rows;
                    const int page_index = key >> page_shift;
                    const int rel = page_index - page_base;
                    int page = rel < FA_TABLE ? page_cache[rel] : table[page_index];
                    if ((unsigned)page >= (unsigned)num_pages) page = 0;
                    const int row = (page * kv_heads + g) * page_size + (key & (page_size - 1));
                    const uint32_t off = (uint32_t)(s * FA_TILE_BYTES + h * FA_HALF_TILE + pg * box_rows * 128);
                    fa_tma_2d(fa_smem(which ? v_stage : k_stage) + off, which ? &map_v : &map_k, h * 64, row, bar);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------------ MMA issuer
        if (lane == 0 && num_tiles > 0) {
            // float32 accumulate, bfloat16 operands, M = 128, N = 64; for P V the second operand is MN-major
            const uint32_t idesc_qk = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(FA_BN >> 3) << 17) | ((uint32_t)(FA_BM >> 4) << 24);
            bool ok = fa_wait(fa_smem(&bars->q_full), 0);
            if (!ok) atomicExch(error_flag, 12);
            auto issue_qk = [&](int j) -> bool {
                const int s = j % FA_STAGES, b = j & 1;
                if (!fa_wait(fa_smem(&bars->kv_full[s]), (j / FA_STAGES) & 1)) return false;
                if (j >= 2 && !fa_wait(fa_smem(P_ALIAS ? &bars->p_free[b] : &bars->s_empty[b]), ((j >> 1) - 1) & 1)) return false;
                fa_fence_after();
                const uint32_t qa = fa_smem(q_tile), ka = fa_smem(k_stage) + s * FA_TILE_BYTES;
#pragma unroll
                for (int k = 0; k < HD / 16; ++k)
                    fa_mma(tmem_base + b * FA_BN, fa_desc(qa + (k >> 2) * FA_ROWS_TILE + (k & 3) * 32),
                           fa_desc(ka + (k >> 2) * FA_HALF_TILE + (k & 3) * 32), idesc_qk, k > 0 ? 1u : 0u);
                fa_commit(fa_smem(&bars->s_full[b]));
                return true;
            };
            for (int j = 0; j < num_tiles && ok; ++j)
                if (!issue_qk(j)) { atomicExch(error_flag, 13); ok = false; }
        }
    } else if (warp == 6) {
        // ------------------------------------------------------------------ issuer of the second product
        if (lane == 0 && num_tiles > 0) {
            const uint32_t idesc_pv = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((uint32_t)(64 >> 3) << 17) | ((uint32_t)(FA_BM >> 4) << 24);
            bool ok = true;
            for (int j = 0; j < num_tiles && ok; ++j) {
                if (!fa_wait(fa_smem(&bars->p_full[j % NP]), (j / NP) & 1)) { atomicExch(error_flag, 14); ok = false; break; }
                fa_fence_after();
                const int s = j % FA_STAGES;
                const uint32_t va = fa_smem(v_stage) + s * FA_TILE_BYTES;
                const uint32_t pa = tmem_base + (P_ALIAS ? (j & 1) * FA_BN : FA_P_COL + (j & 1) * 32);
#pragma unroll
                for (int h = 0; h < HALVES; ++h)
#pragma unroll
                    for (int k = 0; k < FA_BN / 16; ++k)
                        fa_mma_ts(tmem_o + h * 64, pa + k * 8, fa_desc(va + h * FA_HALF_TILE + k * 16 * 128), idesc_pv,
                                  (j > 0 || k > 0) ? 1u : 0u);
                fa_commit(fa_smem(&bars->kv_empty[s]));
                fa_commit(fa_smem(&bars->p_free[j % NP]));
            }
        }
    } else {
        // ------------------------------------------------------------------ softmax and epilogue: one row per thread
        pdl_launch_dependents();
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const int qpos = q_first + row / rep;
        const uint32_t lane_base = tmem_base + ((uint32_t)(quarter * 32) << 16);
        float row_max = -INFINITY, row_sum = 0.f;
        bool ok = true;
        for (int j = 0; j < num_tiles && ok; ++j) {
            const int b = j & 1, s = j % FA_STAGES;
            if (!fa_wait(fa_smem(&bars->s_full[b]), (j >> 1) & 1)) { ok = false; break; }
            fa_fence_after();
            uint32_t raw[2][32];
            fa_ld32(lane_base + b * FA_BN, raw[0]);
            fa_ld32(lane_base + b * FA_BN + 32, raw[1]);
            fa_wait_ld();
            fa_fence_before();
            __syncwarp();
            if (lane == 0) fa_arrive(fa_smem(&bars->s_empty[b]));
            float sc[64];
#pragma unroll
            for (int c = 0; c < 64; ++c) sc[c] = __uint_as_float(raw[c >> 5][c & 31]);
            const int key0 = k_begin + j * FA_BN;
            const bool cut = key0 + FA_BN - 1 > qpos || key0 + FA_BN > k_end;
            if (cut) {
#pragma unroll
                for (int c = 0; c < 64; ++c)
                    if (key0 + c > qpos || key0 + c >= k_end) sc[c] = -INFINITY;
            }
            float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};     // four chains instead of one of 64
#pragma unroll
            for (int c = 0; c < 64; c += 4) {
                m4[0] = fmaxf(m4[0], sc[c]);
                m4[1] = fmaxf(m4[1], sc[c + 1]);
                m4[2] = fmaxf(m4[2], sc[c + 2]);
                m4[3] = fmaxf(m4[3], sc[c + 3]);
            }
            const float tile_max = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
            // The exponent's reference `row_max` follows the true maximum only when that has moved by more
            // than 2^8: probabilities stay below 256 and O needs rescaling (which has to wait for the P V
            // before) only then. Sum and O use the same reference, so the result is exact all the same.
            float alpha = 1.f;
            const float new_max = fmaxf(row_max, tile_max);
            if (row_max == -INFINITY || (new_max - row_max) * scale_log2 > 8.f) {
                alpha = (row_max == -INFINITY) ? 0.f : fa_exp2((row_max - new_max) * scale_log2);
                row_max = new_max;
            }
            const float neg = (row_max == -INFINITY) ? 0.f : -row_max * scale_log2;
            float s4[4] = {0.f, 0.f, 0.f, 0.f};
            uint32_t packed[32];
#pragma unroll
            for (int c = 0; c < 64; c += 4) {
                const float p0 = fa_exp2(fmaf(sc[c], scale_log2, neg));
                const float p1 = fa_exp2(fmaf(sc[c + 1], scale_log2, neg));
                const float p2 = fa_exp2(fmaf(sc[c + 2], scale_log2, neg));
                const float p3 = fa_exp2(fmaf(sc[c + 3], scale_log2, neg));
                s4[0] += p0; s4[1] += p1; s4[2] += p2; s4[3] += p3;
                __nv_bfloat162 h0 = __floats2bfloat162_rn(p0, p1), h1 = __floats2bfloat162_rn(p2, p3);
                packed[c >> 1] = *reinterpret_cast<uint32_t*>(&h0);
                packed[(c >> 1) + 1] = *reinterpret_cast<uint32_t*>(&h1);
            }
            row_sum = row_sum * alpha + ((s4[0] + s4[1]) + (s4[2] + s4[3]));
            // P buffer j % NP is free once the P V of tile j - NP has completed (where P lies over S, the scores
            // of this tile could not have been written before that)
            if (!P_ALIAS && j >= NP && !fa_wait(fa_smem(&bars->p_free[j % NP]), ((j / NP) - 1) & 1)) { ok = false; break; }
            if (j > 0) {
                const bool moved = alpha != 1.f;
                if (__any_sync(0xffffffffu, moved)) {          // warp-collective: rows whose reference stayed scale by 1
                    // O must hold the P V of tile j - 1 before it is rescaled
                    if (!fa_wait(fa_smem(&bars->p_free[(j - 1) % NP]), ((j - 1) / NP) & 1)) { ok = false; break; }
                    fa_fence_after();
#pragma unroll
                    for (int pair = 0; pair < HD / 64; ++pair) {
                        uint32_t o[2][32];
                        fa_ld32(lane_base + 2 * FA_BN + pair * 64, o[0]);
                        fa_ld32(lane_base + 2 * FA_BN + pair * 64 + 32, o[1]);
                        fa_wait_ld();
#pragma unroll
                        for (int h = 0; h < 2; ++h)
#pragma unroll
                            for (int c = 0; c < 32; ++c) o[h][c] = __float_as_uint(__uint_as_float(o[h][c]) * alpha);
                        fa_st32(lane_base + 2 * FA_BN + pair * 64, o[0]);
                        fa_st32(lane_base + 2 * FA_BN + pair * 64 + 32, o[1]);
                    }
                    fa_wait_st();
                }
            }
            // rows of V from the first invisible key on are zeroed (last tile of the range only)
            const int visible_keys = k_end - key0;
            bool wrote_shared = false;
            if (visible_keys < FA_BN) {
                wrote_shared = true;
                unsigned char* v_tile = v_stage + s * FA_TILE_BYTES;
                for (int i = (warp - 2) * 32 + lane; i < (FA_BN - visible_keys) * 8 * HALVES; i += 128) {
                    const int h = i / ((FA_BN - visible_keys) * 8), rest = i % ((FA_BN - visible_keys) * 8);
                    const int r = visible_keys + rest / 8, c = rest % 8;
                    *reinterpret_cast<uint4*>(v_tile + h * FA_HALF_TILE + r * 128 + ((c ^ (r & 7)) << 4)) = make_uint4(0, 0, 0, 0);
                }
            }
            // P row into tensor memory: column c holds the probabilities of keys 2c and 2c + 1
            fa_st32(lane_base + (P_ALIAS ? b * FA_BN : FA_P_COL + b * 32), packed);
            fa_wait_st();
            if (wrote_shared) fa_fence_async();      // generic-proxy writes become visible to the tensor core's reads
            fa_fence_before();
            __syncwarp();
            if (lane == 0) fa_arrive(fa_smem(&bars->p_full[j % NP]));
        }
        if (!ok && lane == 0) atomicExch(error_flag, 15);
        if (ok && num_tiles > 0 && !fa_wait(fa_smem(&bars->p_free[(num_tiles - 1) % NP]), ((num_tiles - 1) / NP) & 1)) {
            ok = false;
            if (lane == 0) atomicExch(error_flag, 16);
        }
        fa_fence_after();
        // ---- epilogue, 64 columns of the row at a time
        const int token = tok0 + row / rep, head = g * rep + row % rep;
        const size_t row_index = (size_t)(seg_start + token) * heads + head;
        const bool writes = row < valid_rows && ok;
        const float inv = row_sum > 0.f ? 1.f / row_sum : 0.f;
#pragma unroll
        for (int pair = 0; pair < HD / 64; ++pair) {
            float o_row[64];
            if (ok && num_tiles > 0) {
                uint32_t o[2][32];
                fa_ld32(lane_base + 2 * FA_BN + pair * 64, o[0]);
                fa_ld32(lane_base + 2 * FA_BN + pair * 64 + 32, o[1]);
                fa_wait_ld();
#pragma unroll
                for (int c = 0; c < 64; ++c) o_row[c] = __uint_as_float(o[c >> 5][c & 31]);
            } else {
#pragma unroll
                for (int c = 0; c < 64; ++c) o_row[c] = 0.f;
            }
            if (!writes) continue;
            if (num_splits > 1) {
                const size_t slot = row_index * num_splits + split;
                float4* dst = reinterpret_cast<float4*>(partial_o + slot * HD + pair * 64);
#pragma unroll
                for (int c = 0; c < 16; ++c) dst[c] = make_float4(o_row[4 * c], o_row[4 * c + 1], o_row[4 * c + 2], o_row[4 * c + 3]);
                if (pair == 0) {
                    partial_ml[slot * 2] = (row_max == -INFINITY) ? -INFINITY : row_max * scale_log2;
                    partial_ml[slot * 2 + 1] = row_sum;
                }
            } else {
                uint4* dst = reinterpret_cast<uint4*>(out + row_index * HD + pair * 64);
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    uint32_t w[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        __nv_bfloat162 h = __floats2bfloat162_rn(o_row[8 * c + 2 * e] * inv, o_row[8 * c + 2 * e + 1] * inv);
                        w[e] = *reinterpret_cast<uint32_t*>(&h);
                    }
                    dst[c] = make_uint4(w[0], w[1], w[2], w[3]);
                }
            }
        }
        fa_fence_before();
    }
    __syncthreads();
    if (warp == 1) {
        fa_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"((uint32_t)FA_TMEM_COLS) : "memory");
    }
}

// ---------------------------------------------------------------------------- host side
typedef CUresult (*FaEncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                               const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                               CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static FaEncodeFn fa_encode_fn() {
    static FaEncodeFn fn = nullptr;
    static bool looked = false;
    if (!looked) {
        looked = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<FaEncodeFn>(p);
    }
    return fn;
}

TTB_EXPORT int ttb_attention_tcgen05_supports(int heads, int kv_heads, int head_dim, int page_size, int window) {
    if ((head_dim != 64 && head_dim != 128) || window > 0 || kv_heads < 1 || heads % kv_heads) return 0;
    if (heads / kv_heads > 16) return 0;
    if (page_size < 8 || (page_size & (page_size - 1))) return 0;
    return 1;
}

TTB_EXPORT int ttb_attention_tcgen05_tile_rows() { return FA_BM; }

template <int HD>
static int launch_attention_tcgen05(const CUtensorMap& map_q, const CUtensorMap& map_k, const CUtensorMap& map_v, void* out,
                                    const int* cu_seqlens, const int* seg_pos0, const int* block_table, int table_width,
                                    int page_size, const int* qtile_seg, const int* qtile_tok0, int n_qtiles, int heads,
                                    int kv_heads, float scale, int num_splits, float* partial_o, float* partial_ml,
                                    int num_pages, int* status, int* error_flag, cudaStream_t stream) {
    constexpr int halves = HD / 64, stages = HD == 64 ? 3 : 2;
    const size_t smem = (size_t)halves * FA_ROWS_TILE + 2 * (size_t)stages * halves * FA_HALF_TILE + sizeof(FaBars) + 16 +
                        FA_TABLE * sizeof(int);
    static TtbOncePerDevice configured;
    if (configured.pending()) {
        cudaError_t e = cudaFuncSetAttribute(attention_tcgen05_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return (int)e;
        configured.mark();
    }
    int page_shift = 0;
    while ((1 << page_shift) < page_size) ++page_shift;
    dim3 grid(n_qtiles, kv_heads, num_splits);
    ttb_launch(attention_tcgen05_kernel<HD>, grid, dim3(FA_THREADS), smem, stream, map_q, map_k, map_v, (__nv_bfloat16*)out,
               cu_seqlens, seg_pos0, block_table, table_width, page_size, page_shift, qtile_seg, qtile_tok0, heads,
               kv_heads, scale * 1.4426950408889634f, num_splits, partial_o, partial_ml, num_pages, status, error_flag);
    return ttb_launch_status();
}

// qkv [tokens, q_row_stride] bfloat16 (queries first), pages [num_pages, kv_heads, page_size, head_dim] bfloat16.
// qtile_seg / qtile_tok0: the segment and first token of each query tile of 128 / (heads / kv_heads) tokens.
// With num_splits > 1: partial_o [tokens * heads * num_splits * head_dim], partial_ml [tokens * heads * num_splits * 2]
// floats, in the format that attention_mma.cu's merge kernel reads. error_flag: device int, set if a wait gave up.
TTB_EXPORT int ttb_paged_attention_tcgen05(const void* qkv, int q_row_stride, void* out, const int* cu_seqlens,
                                           const int* seg_pos0, const void* key_pages, const void* value_pages,
                                           const int* block_table, int table_width, int page_size,
                                           const int* qtile_seg, const int* qtile_tok0, int n_qtiles, int tokens,
                                           int heads, int kv_heads, int head_dim, float scale, int num_splits,
                                           float* partial_o, float* partial_ml, int num_pages, int* status,
                                           int* error_flag, cudaStream_t stream) {
    if (n_qtiles == 0 || tokens == 0) return TTB_OK;
    if (!qkv || !out || !cu_seqlens || !seg_pos0 || !key_pages || !value_pages || !block_table || !qtile_seg ||
        !qtile_tok0 || !error_flag)
        return TTB_ERR_ARGUMENT;
    if (!ttb_attention_tcgen05_supports(heads, kv_heads, head_dim, page_size, 0)) return TTB_ERR_UNSUPPORTED;
    if (q_row_stride % head_dim || !aligned16(qkv) || !aligned16(key_pages) || !aligned16(value_pages) || !aligned16(out))
        return TTB_ERR_UNSUPPORTED;
    if (num_splits < 1 || num_splits > 65535 || kv_heads > 65535) return TTB_ERR_UNSUPPORTED;
    if (num_splits > 1 && (!partial_o || !partial_ml)) return TTB_ERR_ARGUMENT;
    FaEncodeFn encode = fa_encode_fn();
    if (!encode) return TTB_ERR_UNSUPPORTED;
    const int rep = heads / kv_heads;
    CUtensorMap map_q, map_k, map_v;
    {   // queries: (64 elements, half of the head, head, token)
        cuuint64_t dims[4] = {64, (cuuint64_t)(head_dim / 64), (cuuint64_t)(q_row_stride / head_dim), (cuuint64_t)tokens};
        cuuint64_t strides[3] = {128, (cuuint64_t)head_dim * 2, (cuuint64_t)q_row_stride * 2};
        cuuint32_t box[4] = {64, 1, (cuuint32_t)rep, (cuuint32_t)(FA_BM / rep)};
        cuuint32_t elem[4] = {1, 1, 1, 1};
        if (encode(&map_q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(qkv), dims, strides, box, elem,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return TTB_ERR_UNSUPPORTED;
    }
    for (int which = 0; which < 2; ++which) {   // pages: (head_dim elements, row = (page, kv head, slot)), boxes of 64 columns
        cuuint64_t dims[2] = {(cuuint64_t)head_dim, (cuuint64_t)num_pages * kv_heads * page_size};
        cuuint64_t strides[1] = {(cuuint64_t)head_dim * 2};
        cuuint32_t box[2] = {64, (cuuint32_t)(page_size < FA_BN ? page_size : FA_BN)};
        cuuint32_t elem[2] = {1, 1};
        if (encode(which ? &map_v : &map_k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                   const_cast<void*>(which ? value_pages : key_pages), dims, strides, box, elem,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return TTB_ERR_UNSUPPORTED;
    }
#define FA_ARGS map_q, map_k, map_v, out, cu_seqlens, seg_pos0, block_table, table_width, page_size, qtile_seg, qtile_tok0,  \
                n_qtiles, heads, kv_heads, scale, num_splits, partial_o, partial_ml, num_pages, status, error_flag, stream
    return head_dim == 64 ? launch_attention_tcgen05<64>(FA_ARGS) : launch_attention_tcgen05<128>(FA_ARGS);
#undef FA_ARGS
}
