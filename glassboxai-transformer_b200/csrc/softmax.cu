// softmax.cu -- row softmax (replaces softmaxKernel, transformer.cu:126-166,
// which the reference launches once per head, :839-842).
//
// Per row: one HBM read into registers, max by warp shuffles (seeded with
// -1e30f like the reference), e = expf(x - max) kept in registers, sum by
// shuffles, out = e / sum with IEEE division, one HBM write.  The reference
// makes three reads and two writes of every element.  Because max is exact
// and expf / division are the same CUDA functions, every e is bit-identical
// to the reference's; only the order of the sum differs.
#include "rows.cuh"

namespace gbx {

template <int TPR, int V4>
__global__ void __launch_bounds__(kRowCTA)
softmax_vec_kernel(const float* in, float* out, int64_t rows, int L)
{
    constexpr int RPC = kRowCTA / TPR;
    __shared__ float red[2][kRowCTA / 32];
    const int n4 = L >> 2;
    const int lane = threadIdx.x & (TPR - 1);
    const int grp = threadIdx.x / TPR;

    for (int64_t row0 = (int64_t)blockIdx.x * RPC; row0 < rows; row0 += (int64_t)gridDim.x * RPC) {
        const int64_t row = row0 + grp;
        const bool valid = row < rows;
        const int64_t off = row * L;

        float4 v[V4];
#pragma unroll
        for (int k = 0; k < V4; ++k) {
            const int c = k * TPR + lane;
            v[k] = (valid && c < n4) ? ld_stream(in + off + 4 * c)
                                     : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        }
        float m = -1e30f;
#pragma unroll
        for (int k = 0; k < V4; ++k) m = fmaxf(m, fmaxf(fmaxf(v[k].x, v[k].y), fmaxf(v[k].z, v[k].w)));
        m = row_max<TPR>(m, red[0]);

        float s = 0.0f;
#pragma unroll
        for (int k = 0; k < V4; ++k) {
            if (k * TPR + lane < n4) {
                v[k].x = expf(v[k].x - m);
                v[k].y = expf(v[k].y - m);
                v[k].z = expf(v[k].z - m);
                v[k].w = expf(v[k].w - m);
                s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
            }
        }
        s = row_sum<TPR>(s, red[1]);

        if (valid) {
#pragma unroll
            for (int k = 0; k < V4; ++k) {
                const int c = k * TPR + lane;
                if (c < n4)
                    st_stream(out + off + 4 * c,
                              make_float4(v[k].x / s, v[k].y / s, v[k].z / s, v[k].w / s));
            }
        }
    }
}

// General path (any L, any alignment, rows longer than the register path):
// one CTA per row, the reference's three passes with shuffle reductions.
__global__ void __launch_bounds__(kRowCTA)
softmax_general_kernel(const float* in, float* out, int64_t rows, int L)
{
    __shared__ float red[2][kRowCTA / 32];
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const float* ir = in + row * L;
        float* orow = out + row * L;
        float m = -1e30f;
        for (int i = threadIdx.x; i < L; i += kRowCTA) m = fmaxf(m, ir[i]);
        m = block_max(m, red[0]);
        float s = 0.0f;
        for (int i = threadIdx.x; i < L; i += kRowCTA) {
            const float e = expf(ir[i] - m);
            orow[i] = e;
            s += e;
        }
        s = block_sum(s, red[1]);
        for (int i = threadIdx.x; i < L; i += kRowCTA) orow[i] = orow[i] / s;
        __syncthreads();
    }
}

template <int TPR, int V4>
static int launch_softmax_vec(const float* in, float* out, int64_t rows, int L, cudaStream_t stream)
{
    auto k = softmax_vec_kernel<TPR, V4>;
    constexpr int RPC = kRowCTA / TPR;
    const int grid = persistent_grid(k, kRowCTA, 0, (rows + RPC - 1) / RPC, 1);
    if (grid < 1) return GBX_ECUDA;
    k<<<grid, kRowCTA, 0, stream>>>(in, out, rows, L);
    return check_launch("gbx_softmax_rows");
}

}  // namespace gbx

using namespace gbx;

extern "C" int gbx_softmax_rows(const float* in, float* out, int64_t rows, int L, gbx_stream_t stream)
{
    if (rows < 0 || L <= 0) return set_error(GBX_EINVAL, "gbx_softmax_rows: rows=%lld L=%d", (long long)rows, L);
    if (rows == 0) return GBX_OK;
    if (!in || !out) return set_error(GBX_EINVAL, "gbx_softmax_rows: null pointer");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    RowShape shape;
    if (L % 4 == 0 && aligned16(in) && aligned16(out) && row_shape(L / 4, &shape)) {
#define GBX_SM_CALL(T, V) launch_softmax_vec<T, V>(in, out, rows, L, s)
        return GBX_ROW_DISPATCH(shape, GBX_SM_CALL, set_error(GBX_ERANGE, "softmax: no shape for L=%d", L));
#undef GBX_SM_CALL
    }
    const int grid = persistent_grid(softmax_general_kernel, kRowCTA, 0, rows, 4);
    if (grid < 1) return GBX_ECUDA;
    softmax_general_kernel<<<grid, kRowCTA, 0, s>>>(in, out, rows, L);
    return check_launch("gbx_softmax_rows");
}
