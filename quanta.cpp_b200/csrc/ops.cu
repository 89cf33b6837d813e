// Ops-level kernels behind the C ABI's qnt_quantize_q8 / qnt_matvec / qnt_matmul (the reference's
// quantize_q8 / MatvecQFn / MatmulQFn, engine/src/ops.h:52-70).
//
// Arithmetic contract (the "cuda" kernel family): every output is
//     acc = 0;  for b in blocks (in order):  acc = acc + (float(s_b) * dw_b) * dx_b
// with s_b the exact int32 block sum and round-to-nearest mul/add, i.e. matvec_q_ref's expression
// (engine/src/ops_ref.cpp:85-120).  matmul gives, per (row, token), the same bits as matvec.
#include "kernels.cuh"
#include "ops.h"

namespace qb {

// ---------------------------------------------------------------- quantize_q8

// x [n_tok][n] -> q [n_tok][n], d [n_tok][n/32].  One warp per 32-block.
__global__ void k_quantize_q8(const float* __restrict__ x, long long n_blocks, int8_t* __restrict__ q,
                              float* __restrict__ d) {
    const long long blk = (long long)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (blk >= n_blocks) return;
    const int lane = threadIdx.x & 31;
    float dd;
    const int8_t v = quantize_lane(x[blk * QK + lane], &dd);
    q[blk * QK + lane] = v;
    if (lane == 0) d[blk] = dd;
}

cudaError_t launch_quantize_q8(const float* x, int n_tok, int n, int8_t* q, float* d, cudaStream_t st) {
    const long long nb = (long long)n_tok * (n / QK);
    if (nb == 0) return cudaSuccess;
    const int per = kThreads / 32;
    k_quantize_q8<<<unsigned((nb + per - 1) / per), kThreads, 0, st>>>(x, nb, q, d);
    return cudaGetLastError();
}

// ---------------------------------------------------------------- matvec (M = 1)

// CTA = `rows_per_cta` consecutive rows of [r0, r1).  Dynamic smem: sx[cols] | sdx[nb] | ssum[nb] | sterm.
template <int DT, int U>
__global__ void __launch_bounds__(kThreads) k_matvec(DMat W, const int8_t* __restrict__ qx, const float* __restrict__ dx,
                                                     int r0, int r1, int rows_per_cta, unsigned cpr_magic,
                                                     float* __restrict__ out) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int cols = W.cols, nb = cols / QK;
    int8_t* sx = reinterpret_cast<int8_t*>(smem);
    float* sdx = reinterpret_cast<float*>(smem + cols);
    int* ssum = reinterpret_cast<int*>(sdx + nb);
    float* sterm = reinterpret_cast<float*>(ssum + nb);
    const int row0 = r0 + blockIdx.x * rows_per_cta;
    const int nrows = min(rows_per_cta, r1 - row0);
    if (nrows <= 0) return;
    RowSlice S;
    const int rb = row_bytes(DT, cols);
    S.wq = W.q + size_t(row0) * rb;
    S.wd = W.d + size_t(row0) * nb;
    S.nrows = nrows;
    S.nb = nb;
    S.cpr = rb / 16;
    S.cpr_magic = cpr_magic;
    S.tstride = term_stride(nb);
    slice_terms<DT, U>(S, sx, sdx, ssum, sterm,
                       [&] { load_quant(qx, dx, cols, sx, sdx, DT == DT_Q4_0 ? ssum : nullptr); });
    __syncthreads();
    for (int r = threadIdx.x; r < nrows; r += blockDim.x) out[row0 + r] = row_sum(sterm + r * S.tstride, nb);
}

constexpr int kMatvecU = 4;

static int matvec_rows_per_cta(int dtype, int cols) {
    const int cpr = row_bytes_host(dtype, cols) / 16;
    int rows = (kThreads * kMatvecU) / cpr;
    if (rows >= 2) rows &= ~1;
    return rows;
}

size_t matvec_smem(int dtype, int cols) {
    const int nb = cols / QK;
    return size_t(cols) + size_t(nb) * 8 + size_t(matvec_rows_per_cta(dtype, cols)) * (nb | 1) * 4;
}

cudaError_t launch_matvec(const DMat& W, const int8_t* qx, const float* dx, int r0, int r1, float* out, cudaStream_t st) {
    if (r1 <= r0) return cudaSuccess;
    const int rpc = matvec_rows_per_cta(W.dtype, W.cols);
    if (rpc < 1) return cudaErrorInvalidValue;
    const unsigned grid = unsigned((r1 - r0 + rpc - 1) / rpc);
    const size_t sm = matvec_smem(W.dtype, W.cols);
    const unsigned magic = div_magic(unsigned(row_bytes_host(W.dtype, W.cols) / 16));
    if (W.dtype == DT_Q8_0) {
        auto k = k_matvec<DT_Q8_0, kMatvecU>;
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
        k<<<grid, kThreads, sm, st>>>(W, qx, dx, r0, r1, rpc, magic, out);
    } else if (W.dtype == DT_Q4_0) {
        auto k = k_matvec<DT_Q4_0, kMatvecU>;
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
        k<<<grid, kThreads, sm, st>>>(W, qx, dx, r0, r1, rpc, magic, out);
    } else {
        return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

// ---------------------------------------------------------------- matmul on CUDA cores (n <= 32 tokens)

// Tile: 16 rows x 32 tokens; warp w owns rows (2w, 2w+1), lane = token.  K is walked in slabs of 8 blocks staged
// in shared memory; each (row, token) accumulator walks the blocks in order, so it equals the matvec bit for bit.
constexpr int kSimtRows = 16, kSimtTok = 32, kSlab = 8;

template <int DT>
__global__ void __launch_bounds__(kThreads) k_matmul_simt(DMat W, const int8_t* __restrict__ qx, const float* __restrict__ dx,
                                                          int n, int r0, int r1, float* __restrict__ out, int ldo) {
    __shared__ __align__(16) int8_t sx[kSimtTok][kSlab * QK + 16];
    __shared__ float sdx[kSimtTok][kSlab + 1];
    __shared__ int ssum[kSimtTok][kSlab + 1];
    const int cols = W.cols, nb = cols / QK, rb = row_bytes(DT, cols);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = blockIdx.y * kSimtTok;
    const int ra = r0 + blockIdx.x * kSimtRows + 2 * warp, rbw = ra + 1;
    const bool va = ra < r1, vb = rbw < r1;
    const int tok = t0 + lane;
    const bool vt = tok < n;
    float acc_a = 0.f, acc_b = 0.f;
    for (int b0 = 0; b0 < nb; b0 += kSlab) {
        const int nbs = min(kSlab, nb - b0);
        __syncthreads();
        // stage x[t0 .. t0+32)[b0*32 .. (b0+nbs)*32) : 16-byte pieces
        for (int i = threadIdx.x; i < kSimtTok * nbs * 2; i += blockDim.x) {
            const int t = i / (nbs * 2), piece = i - t * nbs * 2;
            int4 v = make_int4(0, 0, 0, 0);
            if (t0 + t < n) v = *reinterpret_cast<const int4*>(qx + size_t(t0 + t) * cols + size_t(b0) * QK + piece * 16);
            *reinterpret_cast<int4*>(&sx[t][piece * 16]) = v;
        }
        for (int i = threadIdx.x; i < kSimtTok * nbs; i += blockDim.x) {
            const int t = i / nbs, bb = i - t * nbs;
            sdx[t][bb] = t0 + t < n ? dx[size_t(t0 + t) * nb + b0 + bb] : 0.f;
        }
        __syncthreads();
        if (DT == DT_Q4_0) {
            for (int i = threadIdx.x; i < kSimtTok * nbs; i += blockDim.x) {
                const int t = i / nbs, bb = i - t * nbs;
                int s = 0;
                for (int k = 0; k < QK; ++k) s += sx[t][bb * QK + k];
                ssum[t][bb] = s;
            }
            __syncthreads();
        }
        for (int bb = 0; bb < nbs; ++bb) {
            const int b = b0 + bb;
            const int8_t* xs = &sx[lane][bb * QK];
            int sa = 0, sb = 0;
            if (DT == DT_Q8_0) {
                const uint4* pa = reinterpret_cast<const uint4*>(W.q + size_t(va ? ra : r0) * rb + size_t(b) * QK);
                const uint4* pb = reinterpret_cast<const uint4*>(W.q + size_t(vb ? rbw : r0) * rb + size_t(b) * QK);
                sa = chunk_dot<DT_Q8_0>(pa[0], xs, 0) + chunk_dot<DT_Q8_0>(pa[1], xs, 1);
                sb = chunk_dot<DT_Q8_0>(pb[0], xs, 0) + chunk_dot<DT_Q8_0>(pb[1], xs, 1);
            } else {
                const uint4* pa = reinterpret_cast<const uint4*>(W.q + size_t(va ? ra : r0) * rb + size_t(b) * 16);
                const uint4* pb = reinterpret_cast<const uint4*>(W.q + size_t(vb ? rbw : r0) * rb + size_t(b) * 16);
                sa = chunk_dot<DT_Q4_0>(pa[0], xs, 0) - 8 * ssum[lane][bb];
                sb = chunk_dot<DT_Q4_0>(pb[0], xs, 0) - 8 * ssum[lane][bb];
            }
            const float d = sdx[lane][bb];
            if (va) acc_a = fadd(acc_a, block_term(sa, __half2float(W.d[size_t(ra) * nb + b]), d));
            if (vb) acc_b = fadd(acc_b, block_term(sb, __half2float(W.d[size_t(rbw) * nb + b]), d));
        }
    }
    if (vt && va) out[size_t(tok) * ldo + ra] = acc_a;
    if (vt && vb) out[size_t(tok) * ldo + rbw] = acc_b;
}

cudaError_t launch_matmul_simt(const DMat& W, const int8_t* qx, const float* dx, int n, int r0, int r1, float* out, int ldo,
                               cudaStream_t st) {
    if (r1 <= r0 || n <= 0) return cudaSuccess;
    dim3 grid(unsigned((r1 - r0 + kSimtRows - 1) / kSimtRows), unsigned((n + kSimtTok - 1) / kSimtTok));
    if (W.dtype == DT_Q8_0) k_matmul_simt<DT_Q8_0><<<grid, kThreads, 0, st>>>(W, qx, dx, n, r0, r1, out, ldo);
    else if (W.dtype == DT_Q4_0) k_matmul_simt<DT_Q4_0><<<grid, kThreads, 0, st>>>(W, qx, dx, n, r0, r1, out, ldo);
    else return cudaErrorInvalidValue;
    return cudaGetLastError();
}

}  // namespace qb
