// Paged attention for decode steps: few query rows (a token's heads of one KV group, up to 16
// rows) against a long run of cached keys. bfloat16 operands, float32 scores, running maximum,
// sum and output in float32; head sizes 64 and 128; page sizes that are powers of two from 8 on.
//
// Against the general tensor-core kernel (attention_mma.cu) two things change.
//  1. The products are transposed: S^T = K Q^T and O^T = V^T P^T. Keys run along the M side of
//     mma.m16n8k16 and the query rows along its N side of 8, so eight query rows cost one
//     instruction per 16 keys and k-step where the untransposed form pays two for sixteen rows
//     of which most are padding. P^T leaves the first product as an accumulator fragment and
//     enters the second as a B fragment; movmatrix transposes its 8 x 8 blocks between the two.
//  2. Keys and values come by TMA, one box of a page's rows (64 elements wide, 128-byte swizzle)
//     per copy, issued by a producer warp that runs STAGES tiles ahead; the four consumer warps
//     wait on the tile's "full" mbarrier and hand the stage back through its "empty" mbarrier.
//     No thread computes addresses for 16-byte copies and no block-wide barrier sits in the loop.
//
// A tile is 64 keys; consumer warp w owns keys 16 w .. 16 w + 15 of every tile for both products
// and keeps its own running maximum, sum and output; the four are merged through shared memory at
// the end. With num_splits > 1 block z takes the z-th chunk of the keys and writes unnormalised
// partial results in the format of attention_mma.cu's merge kernel.
//
// TMA copies whole boxes, so a tile may bring rows that the queries must not see: slots of the
// last page that hold nothing yet, or keys that a window has passed. Their scores are replaced
// by -inf before the softmax; their value rows are zeroed in shared memory before the second
// product, because 0 * x is not 0 for every bit pattern a stale row may hold.
//
// No load uses cluster multicast. Waits on mbarriers are bounded: a role that gives up records a
// code in *error_flag and the block runs to its end (its result is then invalid and the host
// raises).
#include <cuda.h>

#include "common.cuh"

#define AD_BN 64                 // keys per tile
#define AD_CONSUMERS 4           // consumer warps, 16 keys of each tile apiece
#define AD_THREADS ((AD_CONSUMERS + 1) * 32)
#define AD_TABLE_CACHE 1024      // block-table entries kept in shared memory per block
#define AD_WAIT_LIMIT (1u << 22)
#define AD_ERR_PRODUCER 21
#define AD_ERR_CONSUMER 22

__device__ __forceinline__ uint32_t ad_smem(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void ad_mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void ad_mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void ad_mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool ad_mbar_wait(uint32_t bar, uint32_t parity) {
    for (uint32_t i = 0; i < AD_WAIT_LIMIT; ++i) {
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
__device__ __forceinline__ void ad_tma_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(dst), "l"(map), "r"(c0), "r"(c1), "r"(bar) : "memory");
}
// A float at the same shared-memory offset in the block of rank `rank` of this cluster.
__device__ __forceinline__ float ad_ld_cluster(uint32_t local_addr, int rank) {
    uint32_t remote;
    float v;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
    return v;
}
__device__ __forceinline__ void ad_ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ad_ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
// The 8 x 8 block of 16-bit values that the warp holds in accumulator layout, transposed.
__device__ __forceinline__ uint32_t ad_movmatrix_trans(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(y) : "r"(x));
    return y;
}
__device__ __forceinline__ void ad_mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ float ad_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ uint32_t ad_pack(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}
// Byte offset of element column 8 * chunk of key row `row` in a K or V tile: halves of 64 columns,
// each [64 rows][128 bytes] as TMA's 128-byte swizzle leaves it (16-byte chunk index xor row mod 8).
__device__ __forceinline__ uint32_t ad_kv_offset(int row, int chunk) {
    return (uint32_t)((chunk >> 3) * (AD_BN * 128) + row * 128 + (((chunk & 7) ^ (row & 7)) << 4));
}

// NT: query rows in blocks of eight (1 or 2).
template <int HD, int NT, int STAGES>
__global__ void __launch_bounds__(AD_THREADS)
attention_decode_kernel(const __grid_constant__ CUtensorMap map_k, const __grid_constant__ CUtensorMap map_v,
                        const __nv_bfloat16* __restrict__ qkv, int q_row_stride, __nv_bfloat16* __restrict__ out,
                        const int* __restrict__ cu_seqlens, const int* __restrict__ seg_pos0,
                        const int* __restrict__ block_table, int table_width, int page_size, int page_shift,
                        int heads, int kv_heads, float scale_log2, int window, int num_splits,
                        float* __restrict__ partial_o, float* __restrict__ partial_ml, int num_pages,
                        int* __restrict__ status, int* __restrict__ error_flag, int cluster_merge) {
    constexpr int ROWS = 8 * NT;                 // query rows of the tile
    constexpr int CHUNKS = HD / 8;               // 16-byte chunks per row
    constexpr int HALVES = HD / 64;
    constexpr int KS = HD / 16;                  // k-steps of K Q^T
    constexpr int MT = HD / 16;                  // 16-row blocks of O^T
    constexpr int KV_BYTES = AD_BN * HD * 2;     // one tile of keys (or values)
    constexpr int STAGE_BYTES = 2 * KV_BYTES;

    extern __shared__ unsigned char ad_raw[];
    unsigned char* stages = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(ad_raw) + 1023) & ~(uintptr_t)1023);
    unsigned char* q_tile = stages + STAGES * STAGE_BYTES;                     // [ROWS][HD], chunks swizzled by row
    int* page_cache = reinterpret_cast<int*>(q_tile + ROWS * HD * 2);          // [AD_TABLE_CACHE]
    uint64_t* bars = reinterpret_cast<uint64_t*>(page_cache + AD_TABLE_CACHE); // full[STAGES], empty[STAGES]
    const uint32_t full0 = ad_smem(bars), empty0 = ad_smem(bars + STAGES);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int gid = lane >> 2, tig = lane & 3;
    const int seg = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
    const int rep = heads / kv_heads;

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            ad_mbar_init(full0 + 8 * s, 1);
            ad_mbar_init(empty0 + 8 * s, AD_CONSUMERS);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    // The step's metadata (segment bounds, positions, block table) comes from the host, not from the kernel
    // before this one, and the same holds for every key below the first new token's position: all of that is
    // read before pdl_wait(), while the preceding kernel may still be running. The queries and the new
    // tokens' keys and values are that kernel's output and are read after it.
    const int seg_start = cu_seqlens[seg];
    const int seg_tokens = cu_seqlens[seg + 1] - seg_start;
    if (seg_tokens <= 0) return;                                // a padded segment of a captured step
    const int pos0 = seg_pos0[seg];
    const int tile_tokens = min(ROWS / rep, seg_tokens);
    const int valid_rows = tile_tokens * rep;
    const int q_first = pos0, q_last = q_first + tile_tokens - 1;
    const int lo = (window > 0 && q_first - window + 1 > 0) ? q_first - window + 1 : 0;
    const int lo_tile = lo & ~(AD_BN - 1);                      // tiles start on page boundaries
    const int total = q_last - lo_tile + 1;
    const int chunk = ((total + num_splits - 1) / num_splits + AD_BN - 1) / AD_BN * AD_BN;
    const int k_begin = lo_tile + split * chunk;
    const int k_end = min(q_last + 1, k_begin + chunk);
    const int num_tiles = k_begin < k_end ? (k_end - k_begin + AD_BN - 1) / AD_BN : 0;
    const int* table = block_table + (size_t)seg * table_width;
    const int page_base = k_begin >> page_shift;
    const int last_page = num_tiles > 0 ? (k_end - 1) >> page_shift : page_base;

    if (num_tiles > 0) {
        // the block-table entries of this block's keys
        const int count = min(last_page - page_base + 1, AD_TABLE_CACHE);
        for (int i = tid; i < count; i += AD_THREADS) page_cache[i] = table[page_base + i];
    }
    __syncthreads();

    float o_acc[MT][NT][4];
    float col_max[NT][2], col_sum[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        col_max[nt][0] = col_max[nt][1] = -INFINITY;
        col_sum[nt][0] = col_sum[nt][1] = 0.f;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int j = 0; j < 4; ++j) o_acc[mt][nt][j] = 0.f;
    }

    if (warp == AD_CONSUMERS) {
        // ------------------------------------------------------------------ producer
        const int box_rows = min(page_size, AD_BN);
        const int boxes = AD_BN / box_rows;                     // boxes per tile and half, for keys or for values
        const int copies = 2 * boxes * HALVES;                  // <= 32: one lane each
        const int which = lane / (boxes * HALVES);              // 0 keys, 1 values
        const int box = (lane / HALVES) % boxes, half = lane % HALVES;
        bool waited = false;
        for (int tile = 0; tile < num_tiles; ++tile) {
            const int stage = tile % STAGES, round = tile / STAGES;
            if (!waited && k_begin + (tile + 1) * AD_BN > q_first) {      // this tile holds keys of the new tokens
                pdl_wait();
                waited = true;
            }
            if (round > 0 && !ad_mbar_wait(empty0 + 8 * stage, (round - 1) & 1)) {
                if (lane == 0) atomicExch(error_flag, AD_ERR_PRODUCER);
                break;
            }
            if (lane == 0) ad_mbar_expect_tx(full0 + 8 * stage, STAGE_BYTES);
            __syncwarp();
            if (lane < copies) {
                const int key0 = k_begin + tile * AD_BN + box * box_rows;
                // a box past the last key repeats the last page: its rows are masked and zeroed
                const int page_index = min(key0 >> page_shift, last_page);
                const int in_page = (key0 >> page_shift) <= last_page ? (key0 & (page_size - 1)) : 0;
                const int rel = page_index - page_base;
                int page = rel < AD_TABLE_CACHE ? page_cache[rel] : table[page_index];
                if ((unsigned)page >= (unsigned)num_pages) {    // a page id outside the pool: do not follow it, say so
                    if (status != nullptr) atomicExch(status, 0x2000000 + seg);
                    page = 0;
                }
                const int row = (page * kv_heads + kvh) * page_size + in_page;
                const uint32_t dst = ad_smem(stages + stage * STAGE_BYTES + which * KV_BYTES + half * (AD_BN * 128) +
                                             box * box_rows * 128);
                ad_tma_2d(dst, which ? &map_v : &map_k, half * 64, row, full0 + 8 * stage);
            }
        }
        if (!waited) pdl_wait();        // this warp takes part in writing the result
    } else {
        // ------------------------------------------------------------------ consumers
        pdl_wait();
      if (num_tiles > 0) {
        // the query rows (rows beyond valid_rows are zero)
        for (int idx = tid; idx < ROWS * CHUNKS; idx += AD_CONSUMERS * 32) {
            const int r = idx / CHUNKS, c = idx % CHUNKS;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (r < valid_rows) {
                const int token = r / rep, head = kvh * rep + r % rep;
                v = *reinterpret_cast<const uint4*>(qkv + (size_t)(seg_start + token) * q_row_stride + (size_t)head * HD + c * 8);
            }
            *reinterpret_cast<uint4*>(q_tile + r * HD * 2 + ((c ^ (r & 7)) << 4)) = v;
        }
        asm volatile("bar.sync 1, %0;" ::"n"(AD_CONSUMERS * 32) : "memory");      // the consumer warps only
        // B fragments of Q^T: ldmatrix of query rows (lane & 7) at four consecutive chunks gives two k-steps
        uint32_t q_frag[NT][KS][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int k2 = 0; k2 < KS / 2; ++k2) {
                uint32_t r[4];
                const int row = nt * 8 + (lane & 7), c = k2 * 4 + (lane >> 3);
                ad_ldmatrix_x4(r, ad_smem(q_tile + row * HD * 2 + ((c ^ (row & 7)) << 4)));
                q_frag[nt][2 * k2][0] = r[0]; q_frag[nt][2 * k2][1] = r[1];
                q_frag[nt][2 * k2 + 1][0] = r[2]; q_frag[nt][2 * k2 + 1][1] = r[3];
            }
        // the positions of the query rows in this thread's columns
        int qpos[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int j = 0; j < 2; ++j) qpos[nt][j] = q_first + min(nt * 8 + 2 * tig + j, valid_rows - 1) / rep;

        for (int tile = 0; tile < num_tiles; ++tile) {
            const int stage = tile % STAGES;
            if (!ad_mbar_wait(full0 + 8 * stage, (tile / STAGES) & 1)) {
                if (lane == 0) atomicExch(error_flag, AD_ERR_CONSUMER);
                break;
            }
            const uint32_t k_tile = ad_smem(stages + stage * STAGE_BYTES), v_tile = k_tile + KV_BYTES;
            const int key_base = k_begin + tile * AD_BN + warp * 16;

            // ---- S^T = K Q^T: 16 keys x ROWS
            float s[NT][4];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int j = 0; j < 4; ++j) s[nt][j] = 0.f;
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                uint32_t a[4];
                ad_ldmatrix_x4(a, k_tile + ad_kv_offset(warp * 16 + (lane & 15), ks * 2 + (lane >> 4)));
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) ad_mma(s[nt], a, q_frag[nt][ks][0], q_frag[nt][ks][1]);
            }
            // ---- mask, only in tiles that the causal edge, the end of the range or a window cuts
            const int last_key = key_base + 15;
            const bool ragged = last_key >= k_end || key_base < lo;        // rows that no query may see
            if (last_key > q_first || ragged || (window > 0 && key_base <= q_last - window)) {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int key = key_base + gid + ((j >> 1) << 3);
                        const int qp = qpos[nt][j & 1];
                        const bool visible = key < k_end && key <= qp && (window <= 0 || key > qp - window);
                        if (!visible) s[nt][j] = -INFINITY;
                    }
                if (ragged) {
                    for (int idx = lane; idx < 16 * CHUNKS; idx += 32) {
                        const int r = idx / CHUNKS, c = idx % CHUNKS, key = key_base + r;
                        if (key >= k_end || key < lo)
                            asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};"
                                         ::"r"(v_tile + ad_kv_offset(warp * 16 + r, c)), "r"(0) : "memory");
                    }
                    __syncwarp();
                }
            }
            // ---- running maximum and sum per query row (a column here); scores stay unscaled, the
            //      scale goes into the exponent's multiply-add
            uint32_t p_frag[NT][2];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                float alpha[2], neg_max_scaled[2];
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    float m = fmaxf(s[nt][j], s[nt][j + 2]);
                    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
                    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
                    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
                    const float new_max = fmaxf(col_max[nt][j], m);
                    alpha[j] = (col_max[nt][j] == -INFINITY) ? 0.f : ad_exp2((col_max[nt][j] - new_max) * scale_log2);
                    col_max[nt][j] = new_max;
                    neg_max_scaled[j] = (new_max == -INFINITY) ? 0.f : -new_max * scale_log2;
                }
                s[nt][0] = ad_exp2(fmaf(s[nt][0], scale_log2, neg_max_scaled[0]));
                s[nt][1] = ad_exp2(fmaf(s[nt][1], scale_log2, neg_max_scaled[1]));
                s[nt][2] = ad_exp2(fmaf(s[nt][2], scale_log2, neg_max_scaled[0]));
                s[nt][3] = ad_exp2(fmaf(s[nt][3], scale_log2, neg_max_scaled[1]));
                col_sum[nt][0] = fmaf(col_sum[nt][0], alpha[0], s[nt][0] + s[nt][2]);
                col_sum[nt][1] = fmaf(col_sum[nt][1], alpha[1], s[nt][1] + s[nt][3]);
                if (alpha[0] != 1.f || alpha[1] != 1.f) {       // the maximum moved: rescale what was gathered
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                        o_acc[mt][nt][0] *= alpha[0];
                        o_acc[mt][nt][1] *= alpha[1];
                        o_acc[mt][nt][2] *= alpha[0];
                        o_acc[mt][nt][3] *= alpha[1];
                    }
                }
                // P^T as B fragments: keys 0-7 and 8-15 of the warp's sixteen, each block transposed
                p_frag[nt][0] = ad_movmatrix_trans(ad_pack(s[nt][0], s[nt][1]));
                p_frag[nt][1] = ad_movmatrix_trans(ad_pack(s[nt][2], s[nt][3]));
            }
            // ---- O^T += V^T P^T
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                uint32_t a[4];
                ad_ldmatrix_x4_trans(a, v_tile + ad_kv_offset(warp * 16 + (lane & 7) + ((lane >> 4) << 3),
                                                              mt * 2 + ((lane >> 3) & 1)));
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) ad_mma(o_acc[mt][nt], a, p_frag[nt][0], p_frag[nt][1]);
            }
            // ---- the stage goes back to the producer
            if (ragged) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) ad_mbar_arrive(empty0 + 8 * stage);
        }
      }
    }

    pdl_launch_dependents();     // the streaming part is over: the next kernel may move in
    __syncthreads();             // every copy that was issued has been waited for: the stages are free
    float* merge_o = reinterpret_cast<float*>(stages);                          // [consumer][ROWS][HD]
    float* merge_ml = merge_o + AD_CONSUMERS * ROWS * HD;                       // [consumer][ROWS][2]
    if (warp < AD_CONSUMERS) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                float sum = col_sum[nt][j];
                sum += __shfl_xor_sync(0xffffffffu, sum, 4);
                sum += __shfl_xor_sync(0xffffffffu, sum, 8);
                sum += __shfl_xor_sync(0xffffffffu, sum, 16);
                const int row = nt * 8 + 2 * tig + j;
                if (gid == 0) {
                    // from here on the maxima are in the exponent's units (scaled, base 2)
                    merge_ml[(warp * ROWS + row) * 2] = col_max[nt][j] == -INFINITY ? -INFINITY : col_max[nt][j] * scale_log2;
                    merge_ml[(warp * ROWS + row) * 2 + 1] = sum;
                }
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    merge_o[(warp * ROWS + row) * HD + mt * 16 + gid] = o_acc[mt][nt][j];
                    merge_o[(warp * ROWS + row) * HD + mt * 16 + gid + 8] = o_acc[mt][nt][j + 2];
                }
            }
    }
    __syncthreads();
    // With key splits and cluster_merge, the blocks of one (segment, KV head) are one thread-block cluster:
    // each leaves its result in its own shared memory and the rows are finished by reading the others'
    // through distributed shared memory; no partial results in global memory and no merge kernel.
    float* blk_o = merge_ml + AD_CONSUMERS * ROWS * 2;                          // [ROWS][HD]
    float* blk_ml = blk_o + ROWS * HD;                                          // [ROWS][2]
    const bool in_cluster = num_splits > 1 && cluster_merge != 0;
    for (int idx = tid; idx < ROWS * HD; idx += AD_THREADS) {
        const int r = idx / HD, c = idx % HD;
        if (r >= valid_rows) continue;
        float m = -INFINITY;
#pragma unroll
        for (int w = 0; w < AD_CONSUMERS; ++w) m = fmaxf(m, merge_ml[(w * ROWS + r) * 2]);
        float sum = 0.f, o = 0.f;
#pragma unroll
        for (int w = 0; w < AD_CONSUMERS; ++w) {
            const float mw = merge_ml[(w * ROWS + r) * 2];
            const float f = (mw == -INFINITY) ? 0.f : exp2f(mw - m);
            sum += f * merge_ml[(w * ROWS + r) * 2 + 1];
            o += f * merge_o[(w * ROWS + r) * HD + c];
        }
        const int token = r / rep, head = kvh * rep + r % rep;
        const size_t row_index = (size_t)(seg_start + token) * heads + head;
        if (in_cluster) {
            blk_o[r * HD + c] = o;
            if (c == 0) { blk_ml[r * 2] = m; blk_ml[r * 2 + 1] = sum; }
        } else if (num_splits > 1) {
            const size_t slot = row_index * num_splits + split;
            partial_o[slot * HD + c] = o;
            if (c == 0) { partial_ml[slot * 2] = m; partial_ml[slot * 2 + 1] = sum; }
        } else {
            out[row_index * HD + c] = __float2bfloat16_rn(sum > 0.f ? o / sum : 0.f);
        }
    }
    if (in_cluster) {
        // every thread of every block of the cluster comes here (the early return above is taken by all of a
        // cluster's blocks or by none: they share the segment)
        asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
        // row r is finished by the block of rank r mod num_splits
        for (int r = split; r < valid_rows; r += num_splits) {
            const int token = r / rep, head = kvh * rep + r % rep;
            const size_t row_index = (size_t)(seg_start + token) * heads + head;
            for (int c = tid; c < HD; c += AD_THREADS) {
                const uint32_t ml_local = ad_smem(blk_ml + r * 2), o_local = ad_smem(blk_o + r * HD + c);
                float m = -INFINITY;
                for (int s2 = 0; s2 < num_splits; ++s2) m = fmaxf(m, ad_ld_cluster(ml_local, s2));
                float sum = 0.f, o = 0.f;
                for (int s2 = 0; s2 < num_splits; ++s2) {
                    const float ms = ad_ld_cluster(ml_local, s2);
                    if (ms == -INFINITY) continue;
                    const float f = exp2f(ms - m);
                    sum += f * ad_ld_cluster(ml_local + 4, s2);
                    o += f * ad_ld_cluster(o_local, s2);
                }
                out[row_index * HD + c] = __float2bfloat16_rn(sum > 0.f ? o / sum : 0.f);
            }
        }
        // nobody leaves while its shared memory may still be read
        asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    }
}

// ---------------------------------------------------------------------------- host side
typedef CUresult (*AdEncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                               const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                               CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static AdEncodeFn ad_encode_fn() {
    static AdEncodeFn fn = nullptr;
    static bool looked = false;
    if (!looked) {
        looked = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<AdEncodeFn>(p);
    }
    return fn;
}

// Whether this kernel takes the geometry: `rows` query rows per segment (tokens x heads per KV head).
TTB_EXPORT int ttb_attention_decode_supports(int heads, int kv_heads, int head_dim, int page_size, int rows) {
    if (head_dim != 64 && head_dim != 128) return 0;
    if (kv_heads < 1 || heads % kv_heads) return 0;
    if (rows < 1 || rows > 16) return 0;
    if (page_size < 8 || (page_size & (page_size - 1))) return 0;
    return 1;
}

// Blocks that fit one SM at a time (by shared memory): what the host sizes key splits by.
TTB_EXPORT int ttb_attention_decode_blocks_per_sm(int head_dim) { return head_dim == 64 ? 3 : 2; }

extern "C" int ttb_attention_merge(const float* partial_o, const float* partial_ml, void* out, int rows, int num_splits,
                                   int head_dim, cudaStream_t stream);

// Key splits up to this many are merged inside the kernel by a thread-block cluster (16 is the most the
// hardware takes, with the opt-in below); TTB200_CLUSTER_MERGE=0 in the environment turns it off.
#define AD_MAX_CLUSTER 16
static int ad_cluster_limit() {
    static int limit = -1;
    if (limit < 0) {
        const char* e = getenv("TTB200_CLUSTER_MERGE");
        limit = (e && e[0] == '0') ? 0 : AD_MAX_CLUSTER;
    }
    return limit;
}

static int ad_sm_count() {
    static int count = 0;
    if (count == 0) {
        int device = 0;
        cudaGetDevice(&device);
        cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device);
        if (count <= 0) count = 1;
    }
    return count;
}

// Whether a call with this many key splits and blocks (segments x KV heads x splits) needs no partial results
// and no merge kernel. Clusters are placed as a whole, which costs occupancy once the grid is larger than the
// GPU: measured at Llama 3.2 1B geometry and 8,192 keys, the step is 2 to 3 % faster with them at batch 1 and 2
// (128 and 256 blocks) and 5 to 12 % slower at batch 4, 8 and 64 (416 blocks and more).
TTB_EXPORT int ttb_attention_decode_merges_in_kernel(int num_splits, int blocks) {
    return num_splits > 1 && num_splits <= ad_cluster_limit() && blocks <= 2 * ad_sm_count();
}

template <int HD, int NT, int STAGES>
static int launch_attention_decode(const CUtensorMap& map_k, const CUtensorMap& map_v, const void* qkv, int q_row_stride,
                                   void* out, const int* cu_seqlens, const int* seg_pos0, const int* block_table,
                                   int table_width, int page_size, int segments, int heads, int kv_heads, float scale,
                                   int window, int num_splits, float* partial_o, float* partial_ml, int num_pages,
                                   int* status, int* error_flag, cudaStream_t stream) {
    const size_t stage_bytes = (size_t)STAGES * 2 * AD_BN * HD * 2;
    const size_t merge_bytes = (size_t)(AD_CONSUMERS + 1) * 8 * NT * (HD + 2) * sizeof(float);
    const size_t smem = 1024 + (stage_bytes > merge_bytes ? stage_bytes : merge_bytes) + (size_t)8 * NT * HD * 2 +
                        AD_TABLE_CACHE * sizeof(int) + 2 * STAGES * sizeof(uint64_t);
    auto kernel = attention_decode_kernel<HD, NT, STAGES>;
    static TtbOncePerDevice configured;
    if (configured.pending()) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return (int)e;
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) cudaGetLastError();
        configured.mark();
    }
    int page_shift = 0;
    while ((1 << page_shift) < page_size) ++page_shift;
    const bool cluster = ttb_attention_decode_merges_in_kernel(num_splits, segments * kv_heads * num_splits) != 0;
    if (!cluster && num_splits > 1 && (!partial_o || !partial_ml)) return TTB_ERR_ARGUMENT;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(segments, kv_heads, num_splits);
    cfg.blockDim = dim3(AD_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    int n_attr = 0;
    if (ttb_pdl_enabled()) {
        attr[n_attr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n_attr].val.programmaticStreamSerializationAllowed = 1;
        ++n_attr;
    }
    if (cluster) {
        attr[n_attr].id = cudaLaunchAttributeClusterDimension;
        attr[n_attr].val.clusterDim.x = 1;
        attr[n_attr].val.clusterDim.y = 1;
        attr[n_attr].val.clusterDim.z = num_splits;
        ++n_attr;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n_attr;
    cudaLaunchKernelEx(&cfg, kernel, map_k, map_v, (const __nv_bfloat16*)qkv, q_row_stride, (__nv_bfloat16*)out, cu_seqlens,
                       seg_pos0, block_table, table_width, page_size, page_shift, heads, kv_heads,
                       scale * 1.4426950408889634f, window, num_splits, partial_o, partial_ml, num_pages, status, error_flag,
                       cluster ? 1 : 0);
    return ttb_launch_status();
}

// One query tile per segment: all its tokens' heads of a KV group, max_rows = max tokens x heads / kv_heads <= 16.
// qkv [tokens, q_row_stride] bfloat16 (queries first), pages [num_pages, kv_heads, page_size, head_dim] bfloat16.
// With num_splits > 1 and not ttb_attention_decode_merges_in_kernel(num_splits, segments * kv_heads * num_splits): partial_o [tokens * heads *
// num_splits * head_dim] and partial_ml [tokens * heads * num_splits * 2] floats of scratch memory, merged by a second
// kernel that this call launches too. `tokens`: the rows of qkv. status: set on a page id outside the pool;
// error_flag: set if a wait gave up.
TTB_EXPORT int ttb_paged_attention_decode(const void* qkv, int q_row_stride, void* out, const int* cu_seqlens,
                                          const int* seg_pos0, const void* key_pages, const void* value_pages,
                                          const int* block_table, int table_width, int page_size, int segments,
                                          int tokens, int max_rows, int heads, int kv_heads, int head_dim, float scale, int window,
                                          int num_splits, float* partial_o, float* partial_ml, int num_pages,
                                          int* status, int* error_flag, cudaStream_t stream) {
    if (segments == 0) return TTB_OK;
    if (!qkv || !out || !cu_seqlens || !seg_pos0 || !key_pages || !value_pages || !block_table || !error_flag)
        return TTB_ERR_ARGUMENT;
    if (!ttb_attention_decode_supports(heads, kv_heads, head_dim, page_size, max_rows)) return TTB_ERR_UNSUPPORTED;
    if ((q_row_stride & 7) || !aligned16(qkv) || !aligned16(key_pages) || !aligned16(value_pages)) return TTB_ERR_UNSUPPORTED;
    if (num_splits < 1 || num_splits > 65535 || kv_heads > 65535 || num_pages < 1) return TTB_ERR_UNSUPPORTED;
    if ((size_t)num_pages * kv_heads * page_size > 0x7fffffffull) return TTB_ERR_UNSUPPORTED;
    AdEncodeFn encode = ad_encode_fn();
    if (!encode) return TTB_ERR_UNSUPPORTED;
    CUtensorMap map_k, map_v;
    for (int which = 0; which < 2; ++which) {   // pages: (head_dim elements, row = (page, kv head, slot))
        cuuint64_t dims[2] = {(cuuint64_t)head_dim, (cuuint64_t)num_pages * kv_heads * page_size};
        cuuint64_t strides[1] = {(cuuint64_t)head_dim * 2};
        cuuint32_t box[2] = {64, (cuuint32_t)(page_size < AD_BN ? page_size : AD_BN)};
        cuuint32_t elem[2] = {1, 1};
        if (encode(which ? &map_v : &map_k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                   const_cast<void*>(which ? value_pages : key_pages), dims, strides, box, elem,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return TTB_ERR_UNSUPPORTED;
    }
#define AD_ARGS map_k, map_v, qkv, q_row_stride, out, cu_seqlens, seg_pos0, block_table, table_width, page_size, segments, \
                heads, kv_heads, scale, window, num_splits, partial_o, partial_ml, num_pages, status, error_flag, stream
    int code;
    if (head_dim == 64)
        code = max_rows <= 8 ? launch_attention_decode<64, 1, 4>(AD_ARGS) : launch_attention_decode<64, 2, 4>(AD_ARGS);
    else
        code = max_rows <= 8 ? launch_attention_decode<128, 1, 3>(AD_ARGS) : launch_attention_decode<128, 2, 3>(AD_ARGS);
#undef AD_ARGS
    if (code != TTB_OK || num_splits == 1 || ttb_attention_decode_merges_in_kernel(num_splits, segments * kv_heads * num_splits))
        return code;
    return ttb_attention_merge(partial_o, partial_ml, out, tokens * heads, num_splits, head_dim, stream);
}
