// Skinny matrix product for decoding: out[m, n] = sum_k x[m, k] * w[n, k] for a handful of
// rows m (one per decoded token). The weight matrix is streamed once from HBM with 16-byte
// loads; each warp owns ROWS weight rows and all M activations rows, accumulates in float32
// and reduces across its lanes. The order of summation for one (m, n) does not depend on M.
#include "common.cuh"

#define GV_WARPS 4
#define GV_ROWS 2

template <typename T, typename TO, int MAXM>
__global__ void __launch_bounds__(GV_WARPS * 32)
gemv_kernel(const T* __restrict__ x, const T* __restrict__ w, TO* __restrict__ out, int M, int N, int K, int ldx,
            int ldw, int ldo, int vec) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int n0 = (blockIdx.x * GV_WARPS + warp) * GV_ROWS;
    if (n0 >= N) return;
    float acc[GV_ROWS][MAXM];
#pragma unroll
    for (int r = 0; r < GV_ROWS; ++r)
#pragma unroll
        for (int m = 0; m < MAXM; ++m) acc[r][m] = 0.f;
    const T* wrow[GV_ROWS];
#pragma unroll
    for (int r = 0; r < GV_ROWS; ++r) wrow[r] = w + (size_t)(n0 + r < N ? n0 + r : N - 1) * ldw;

    if (vec) {
#pragma unroll 2
        for (int k = lane * 8; k < K; k += 256) {
            float wv[GV_ROWS][8];
#pragma unroll
            for (int r = 0; r < GV_ROWS; ++r) load8(wrow[r] + k, wv[r]);
#pragma unroll
            for (int m = 0; m < MAXM; ++m) {
                if (m < M) {
                    float xv[8];
                    load8(x + (size_t)m * ldx + k, xv);
#pragma unroll
                    for (int r = 0; r < GV_ROWS; ++r)
#pragma unroll
                        for (int e = 0; e < 8; ++e) acc[r][m] = fmaf(xv[e], wv[r][e], acc[r][m]);
                }
            }
        }
    } else {
        for (int k = lane; k < K; k += 32) {
#pragma unroll
            for (int r = 0; r < GV_ROWS; ++r) {
                const float wv = to_float(wrow[r][k]);
#pragma unroll
                for (int m = 0; m < MAXM; ++m)
                    if (m < M) acc[r][m] = fmaf(to_float(x[(size_t)m * ldx + k]), wv, acc[r][m]);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < GV_ROWS; ++r)
#pragma unroll
        for (int m = 0; m < MAXM; ++m) {
            const float total = warp_sum(acc[r][m]);
            if (lane == 0 && m < M && n0 + r < N) out[(size_t)m * ldo + n0 + r] = from_float<TO>(total);
        }
}

template <typename T, typename TO>
static int gemv_dispatch(const void* x, const void* w, void* out, int M, int N, int K, int ldx, int ldw, int ldo,
                         cudaStream_t stream) {
    const int vec = (K % 8 == 0) && (ldx % 8 == 0) && (ldw % 8 == 0) && aligned16(x) && aligned16(w);
    const int blocks = (N + GV_WARPS * GV_ROWS - 1) / (GV_WARPS * GV_ROWS);
#define GV_LAUNCH(MM) gemv_kernel<T, TO, MM><<<blocks, GV_WARPS * 32, 0, stream>>>((const T*)x, (const T*)w, (TO*)out, M, N, K, ldx, ldw, ldo, vec)
    if (M <= 1) GV_LAUNCH(1);
    else if (M <= 2) GV_LAUNCH(2);
    else if (M <= 4) GV_LAUNCH(4);
    else if (M <= 8) GV_LAUNCH(8);
    else return TTB_ERR_UNSUPPORTED;
#undef GV_LAUNCH
    return ttb_launch_status();
}

// M <= 8. in_dtype: x and w; out_dtype: out (float32 out of bfloat16 inputs is allowed).
TTB_EXPORT int ttb_gemv(const void* x, const void* w, void* out, int in_dtype, int out_dtype, int M, int N, int K,
                        int ldx, int ldw, int ldo, cudaStream_t stream) {
    if (M == 0 || N == 0) return TTB_OK;
    if (!x || !w || !out || K < 1) return TTB_ERR_ARGUMENT;
    if (in_dtype == TTB_DTYPE_BF16 && out_dtype == TTB_DTYPE_BF16)
        return gemv_dispatch<__nv_bfloat16, __nv_bfloat16>(x, w, out, M, N, K, ldx, ldw, ldo, stream);
    if (in_dtype == TTB_DTYPE_BF16 && out_dtype == TTB_DTYPE_F32)
        return gemv_dispatch<__nv_bfloat16, float>(x, w, out, M, N, K, ldx, ldw, ldo, stream);
    if (in_dtype == TTB_DTYPE_F32 && out_dtype == TTB_DTYPE_F32)
        return gemv_dispatch<float, float>(x, w, out, M, N, K, ldx, ldw, ldo, stream);
    return TTB_ERR_UNSUPPORTED;
}
