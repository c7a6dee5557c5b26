// gpb2_dense_tri.cu -- triangular kernels of the dense first layer: L*x, L^T*x and the Cholesky
// pullback of generate_grad_vals (src/grad_generate_vals.jl:252-280).
//
// L*x and L^T*x (generate_dense, the dense adjoint of generate_grad_xi) accumulate each output
// from 0 in ascending index with rounded multiplies and adds, the oracle's order, so the dense
// layer's contribution to generate and generate_grad_xi is bit-identical to it.  Each CTA owns 32
// outputs; its other warps stream the factor through shared memory while warp 0 runs the 32
// sequential sums.
//
// The pullback of f = L*xi with cotangent vb is  S = L^-T Phi(L^T Lbar) L^-1  with
// Lbar = tril(vb xi^T) (Phi: lower triangle, halved diagonal).  Because L^T is upper triangular,
// (L^T Lbar)_ij = xi_j * sum_{k >= max(i,j)} L_ki vb_k, which for i >= j is xi_j * u_i with
// u = L^T vb.  So Phi(L^T Lbar) = Phi(tril(u xi^T)) needs one matrix-vector product instead of a
// triangular matrix product, and it is generated on the fly from u and xi.
//
// With A = L^-1 (computed once per factorisation, below) and P = D_u T' D_xi, where T' is the
// lower all-ones matrix with 1/2 on its diagonal,  S = A^T P A = F^T H  with F = D_u A and
// H = T' D_xi A (a running sum down each column of D_xi A, the current term halved): one GEMM
// per call.  A itself is built by recursive doubling from the inverses of the 32x32 diagonal
// blocks: for consecutive diagonal blocks of size s, A21 = -A22 (L21 A11), two strided-batched
// GEMMs per level.  (k_trsm_lt below solves the same problem column-chunk by column-chunk, as
// two triangular solves X = L^-T P, S^T = L^-T X^T; it serves blocks too large for the inverse
// workspace.)
//
// S is then two triangular solves with n right-hand sides:  X = L^-T P  and  S^T = L^-T X^T.
// k_trsm_lt solves L^T X = B for a chunk of NB right-hand-side columns per CTA, by 32-row blocks
// from the bottom: the rows already solved stay in shared memory; the block's right-hand side is
// reduced against them with the factor streamed through a cp.async pipeline of 64-row tiles
// (lanes along the block's 32 columns, warps along the tile's rows), and the block is finished by
// a product with the transposed inverse of its 32x32 diagonal block (computed once per
// factorisation by k_diag_inv, in parallel over blocks), so no step carries a chain of
// divisions.  The output is written transposed, which is the right-hand side of the second solve.
// The pullback is not an exact-order computation (neither is the reference's BLAS); it uses
// fused multiply-adds.
#include <algorithm>

#include <cuda_pipeline_primitives.h>

#include "gpb2_problem.h"

namespace gpb2 {

namespace {

constexpr int kTB = 32;        // diagonal block size
constexpr int kTriThreads = 256;
constexpr int kTriWarps = kTriThreads / 32;
constexpr int kDiagWarps = 4;  // k_diag_inv: blocks per CTA (its staging fits 48 KB in f64)
constexpr int kTileRows = 64;  // rows of the factor per pipeline stage in k_trsm_lt

template <typename T>
__host__ __device__ constexpr int tri_stages() { return sizeof(T) == 4 ? 6 : 4; }

// Pitch of the row-major copy: rows start on 128-byte boundaries (cp.async needs 16).
inline int64_t tri_pitch(int64_t n) { return (n + 31) / 32 * 32; }

// Row-major copy: R[i*ld + j] = L[i][j] = L_colmajor[i + j*n] (lower part; upper zero).
template <typename T>
__global__ void k_transpose_lower(const T* __restrict__ L, T* __restrict__ R, int64_t n,
                                  int64_t ld) {
    __shared__ T tile[32][33];
    const int64_t nb = (n + 31) / 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    for (int64_t t = blockIdx.x; t < nb * nb; t += gridDim.x) {
        const int64_t bi = t / nb, bj = t - bi * nb;  // output tile: rows bi*32.., cols bj*32..
        for (int yy = ty; yy < 32; yy += blockDim.x / 32) {
            const int64_t row = bi * 32 + tx, col = bj * 32 + yy;  // tile[yy][tx] = L[row][col]
            tile[yy][tx] = (row < n && col < n) ? L[row + col * n] : T(0);
        }
        __syncthreads();
        for (int yy = ty; yy < 32; yy += blockDim.x / 32) {
            const int64_t i = bi * 32 + yy, j = bj * 32 + tx;  // R[i][j] = L[i][j]
            if (i < n && j < ld) R[i * ld + j] = (j <= i && j < n) ? tile[tx][yy] : T(0);
        }
        __syncthreads();
    }
}

// Asynchronous element copy global -> shared (cp.async, cached at L1+L2); `in` = false writes
// zero and reads nothing.
template <typename T>
__device__ __forceinline__ void cp_async_elem(T* dst, const T* src, bool in) {
    const unsigned int d = (unsigned int)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.ca.shared.global [%0], [%1], %2, %3;" ::"r"(d), "l"(src),
                 "n"((int)sizeof(T)), "r"(in ? (int)sizeof(T) : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Exact-order L*x (TRANS = false) and L^T*x (TRANS = true), outputs [i0, i0 + 32) per CTA.
//   L x:   y_i = sum_{j=0..i} L[i][j] x_j   (column-major factor: M(i, j) = L[i + j*n])
//   L^T x: y_i = sum_{k=i..n-1} L[k][i] x_k (row-major copy:     M(i, k) = R[k*ld + i])
// Either way term k of output row r is M[k * stride + r].  Each output is one chain of
// additions in the oracle's order, so the kernel is built around warp 0 (lane = output) doing
// nothing but those additions: warps 1.. stream the factor and x through a cp.async pipeline
// of kCh-term chunks, form the rounded products and store them transposed (a row of terms per
// output), from where warp 0 reads 16 bytes of terms per load.  Terms outside the triangle are
// +0, which leaves the running sum unchanged (it starts at +0 and can never become -0).
constexpr int kTrmvThreads = 512;  // warp 0 adds, 15 warps stream and form products
template <typename T, bool TRANS>
__global__ void __launch_bounds__(kTrmvThreads)
k_trmv_exact(const T* __restrict__ M, int64_t ld, const T* __restrict__ x, T* __restrict__ y,
             int64_t n) {
    using N = Num<T>;
    using V = typename std::conditional<sizeof(T) == 4, float4, double2>::type;
    constexpr int kV = 16 / (int)sizeof(T);       // terms per vector load
    constexpr int kCh = 256 / (int)sizeof(T);     // terms per chunk (8 KB of the factor)
    constexpr int kS = 3;                         // chunks of the factor in flight
    constexpr int kP = kCh + kV;                  // row pitch of the product tile
    constexpr int kProd = kTrmvThreads - 32;       // threads of warps 1..
    __shared__ __align__(16) T raw[kS][kCh * 32];
    __shared__ __align__(16) T xs[kS][kCh];
    __shared__ __align__(16) T P[2][32 * kP];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t i0 = (int64_t)blockIdx.x * 32, i = i0 + lane;
    const int64_t lo = TRANS ? i0 : 0;  // summation index range
    const int64_t hi = TRANS ? n : (i0 + 32 < n ? i0 + 32 : n);
    const int64_t nch = (hi - lo + kCh - 1) / kCh;
    const int64_t stride = TRANS ? ld : n;
    // Producer pt (warps 1..) always handles output row ii = pt % 32 and the chunk's terms
    // kk = pt / 32 + kRows * m: kProd is a multiple of 32, so all index arithmetic below is a
    // fixed per-thread offset plus 32-bit steps.
    constexpr int kRows = kProd / 32;
    const int pt = threadIdx.x - 32, ii = pt & 31, kk0 = pt >> 5;
    const int r = (int)i0 + ii;
    const bool r_in = r < n;
    const int hi_i = (int)hi;
    auto issue = [&](int64_t c) {  // producers: their share of chunk c, then one commit
        if (c < nch) {
            T* tb = raw[c % kS] + pt;
            const int k0 = (int)(lo + c * kCh) + kk0;
            const T* src = M + (int64_t)k0 * stride + r;
            const int64_t step = (int64_t)kRows * stride;
#pragma unroll
            for (int m = 0; m * kRows + kk0 < kCh; m++) {
                const bool in = r_in && k0 + m * kRows < hi_i;
                cp_async_elem(tb + m * kProd, in ? src : M, in);
                src += step;
            }
            if (pt < kCh) {
                const int k = (int)(lo + c * kCh) + pt;
                cp_async_elem(xs[c % kS] + pt, k < hi_i ? x + k : x, k < hi_i);
            }
        }
        cp_async_commit();
    };
    auto form = [&](int64_t c) {  // producers: rounded products of chunk c, transposed
        cp_async_wait<kS - 2>();  // this thread's copies of chunk c have landed
        asm volatile("bar.sync 1, %0;" ::"n"(kProd) : "memory");  // everyone's; chunk c-1 formed
        issue(c + kS - 1);
        const T* tb = raw[c % kS] + pt;
        const T* xb = xs[c % kS] + kk0;
        T* pb = P[c & 1] + ii * kP + kk0;
        const int k0 = (int)(lo + c * kCh) + kk0;
#pragma unroll
        for (int m = 0; m * kRows + kk0 < kCh; m++) {
            const int k = k0 + m * kRows;
            const bool valid = k < hi_i && (TRANS ? k >= r : k <= r);
            const T pr = N::mul(tb[m * kProd], xb[m * kRows]);
            pb[m * kRows] = valid ? pr : T(0);
        }
    };
    if (w != 0) {
#pragma unroll
        for (int c = 0; c < kS - 1; c++) issue(c);
        form(0);
    }
    __syncthreads();
    T acc = T(0);
    for (int64_t c = 0; c < nch; c++) {
        if (w == 0) {
            const V* row = reinterpret_cast<const V*>(P[c & 1] + lane * kP);
#pragma unroll 4
            for (int q = 0; q < kCh / kV; q++) {
                const V v = row[q];
                if constexpr (sizeof(T) == 4) {
                    acc = N::add(acc, v.x);
                    acc = N::add(acc, v.y);
                    acc = N::add(acc, v.z);
                    acc = N::add(acc, v.w);
                } else {
                    acc = N::add(acc, v.x);
                    acc = N::add(acc, v.y);
                }
            }
        } else if (c + 1 < nch) {
            form(c + 1);
        }
        __syncthreads();  // chunk c+1's products are ready; chunk c's are consumed
    }
    if (w != 0) cp_async_wait<0>();
    if (w == 0 && i < n) y[i] = acc;
}

// Transposed inverses of the 32x32 diagonal blocks of L: DinvT[b][j][i] = (L_bb^-1)[i][j].
// One warp per block; lane j solves L_bb d = e_j by forward substitution.
template <typename T>
__global__ void k_diag_inv(const T* __restrict__ Lr, int64_t n, int64_t ld,
                           T* __restrict__ DinvT) {
    __shared__ T S[kDiagWarps][kTB][kTB + 1];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t nbk = (n + kTB - 1) / kTB;
    const int64_t b = (int64_t)blockIdx.x * kDiagWarps + w;
    if (b >= nbk) return;  // warp-uniform; no block-wide barrier below
    const int64_t r0 = b * kTB;
    const int bs = (int)(n - r0 < kTB ? n - r0 : kTB);
    for (int i = 0; i < kTB; i++)
        S[w][i][lane] = (i < bs && lane <= i) ? Lr[(r0 + i) * ld + r0 + lane] : T(0);
    __syncwarp();
    T d[kTB] = {};
    sfor<0, kTB>([&](auto i_) {
        GPB2_CI(i);
        T s = (i == lane) ? T(1) : T(0);
        sfor<0, i>([&](auto k_) {
            GPB2_CI(k);
            s = fma(-S[w][i][k], d[k], s);
        });
        d[i] = (i < bs && i >= lane) ? s / S[w][i][i] : T(0);
    });
    T* out = DinvT + b * kTB * kTB + lane * kTB;  // row `lane` of the transposed inverse
    sfor<0, kTB>([&](auto i_) {
        GPB2_CI(i);
        out[i] = d[i];
    });
}

// Solve L^T X = B for the right-hand-side columns [c0, c0 + NB), c0 = blockIdx.x * NB.
//   GEN:  B = Phi(tril(u xi^T)) (generated);  else B = Bin, column-major n x n.
//   Output: Xout[i*n + c] = X[i][c] (X row-major, i.e. X^T column-major).
// Shared memory: Lt[stages][64][32] (factor tiles), Xs[npad][NB] (solved rows),
// Red[warps][NB][32], Rb[32][NB+1], Dt[32][33].
template <typename T, int NB, bool GEN>
__global__ void __launch_bounds__(kTriThreads)
k_trsm_lt(const T* __restrict__ Lr, int64_t ld, const T* __restrict__ DinvT,
          const T* __restrict__ u, const T* __restrict__ xi, const T* __restrict__ Bin,
          T* __restrict__ Xout, int64_t n) {
    constexpr int NS = tri_stages<T>();
    constexpr int kPieces = kTB * (int)sizeof(T) / 16;  // 16-byte pieces per tile row
    constexpr int kPer = 16 / (int)sizeof(T);           // elements per piece
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int64_t nbk = (n + kTB - 1) / kTB, npad = nbk * kTB;
    T* Lt = reinterpret_cast<T*>(smem_raw);  // [NS][64][32]
    T* Xs = Lt + (size_t)NS * kTileRows * kTB;  // [npad][NB]
    T* Red = Xs + npad * NB;                    // [warps][NB][32]
    T (*Rb)[NB + 1] = reinterpret_cast<T (*)[NB + 1]>(Red + kTriWarps * kTB * NB);  // [32][NB+1]
    T (*Dt)[kTB + 1] = reinterpret_cast<T (*)[kTB + 1]>(&Rb[kTB][0]);               // [32][33]
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t c0 = (int64_t)blockIdx.x * NB;

    // Tile stream: blocks I = nbk-2 .. 0, each over rows [32(I+1), n) in 64-row tiles.
    int64_t pI = nbk - 2, pk = (nbk - 1) * kTB;  // producer cursor (next tile to fetch)
    int ptile = 0;                                 // tiles issued (committed groups)
    auto issue = [&]() {
        if (pI >= 0) {
            T* dst = Lt + (size_t)(ptile % NS) * kTileRows * kTB;
            const int64_t r0 = pI * kTB;
            for (int e = threadIdx.x; e < kTileRows * kPieces; e += kTriThreads) {
                const int kk = e / kPieces, q = e % kPieces;
                const int64_t k = pk + kk;
                if (k < n)
                    __pipeline_memcpy_async(dst + kk * kTB + q * kPer,
                                            Lr + k * ld + r0 + q * kPer, 16);
            }
            pk += kTileRows;
            if (pk >= n) {
                pI -= 1;
                pk = (pI + 1) * kTB;
            }
        }
        __pipeline_commit();
        ptile++;
    };
    for (int st = 0; st < NS - 1; st++) issue();
    int ctile = 0;  // tiles consumed

    // Operands of a block's finish (its diagonal inverse and right-hand side), fetched one block
    // ahead so their latency hides behind the previous block's tiles.
    constexpr int kDin = kTB * kTB / kTriThreads;
    constexpr int kRhs = (kTB * NB + kTriThreads - 1) / kTriThreads;
    auto fetch = [&](int64_t I, T (&dreg)[kDin], T (&breg)[kRhs]) {
        const int64_t r0 = I * kTB;
#pragma unroll
        for (int q = 0; q < kDin; q++)
            dreg[q] = DinvT[I * kTB * kTB + threadIdx.x + q * kTriThreads];
#pragma unroll
        for (int q = 0; q < kRhs; q++) {
            const int e = threadIdx.x + q * kTriThreads;
            const int i = e % kTB, c = e / kTB;
            const int64_t gi = r0 + i, gc = c0 + c;
            T b = T(0);
            if (e < kTB * NB && gi < n && gc < n) {
                if (GEN) {
                    const T pr = u[gi] * xi[gc];
                    b = gi > gc ? pr : (gi == gc ? T(0.5) * pr : T(0));
                } else {
                    b = Bin[gi + gc * n];
                }
            }
            breg[q] = b;
        }
    };
    T dreg[kDin], breg[kRhs];
    fetch(nbk - 1, dreg, breg);

    for (int64_t I = nbk - 1; I >= 0; I--) {
        const int64_t r0 = I * kTB, r1 = r0 + kTB < n ? r0 + kTB : n;
        T dnext[kDin], bnext[kRhs];
        if (I > 0) fetch(I - 1, dnext, bnext);
        // (1) partial sums of L[k][r0 + lane] * X[k][c] over the solved rows k >= r1
        T acc[NB];
#pragma unroll
        for (int c = 0; c < NB; c++) acc[c] = T(0);
        for (int64_t k0 = r1; k0 < n; k0 += kTileRows) {
            __pipeline_wait_prior(NS - 2);  // this thread's copies of tile `ctile` have landed
            __syncthreads();                // everyone's; the stage of tile ctile-1 is free
            issue();
            const T* tl = Lt + (ctile % NS) * (kTileRows * kTB) + lane;
            const T* xt = Xs + (int)k0 * NB;
            if (n - k0 >= kTileRows) {
#pragma unroll
                for (int q = 0; q < kTileRows / kTriWarps; q++) {
                    const int kk = w + q * kTriWarps;
                    const T l = tl[kk * kTB];
                    const T* xr = xt + kk * NB;
#pragma unroll
                    for (int c = 0; c < NB; c++) acc[c] = fma(l, xr[c], acc[c]);
                }
            } else {
                const int rows = (int)(n - k0);
                for (int kk = w; kk < rows; kk += kTriWarps) {
                    const T l = tl[kk * kTB];
                    const T* xr = xt + kk * NB;
#pragma unroll
                    for (int c = 0; c < NB; c++) acc[c] = fma(l, xr[c], acc[c]);
                }
            }
            ctile++;
        }
#pragma unroll
        for (int c = 0; c < NB; c++) Red[(w * NB + c) * kTB + lane] = acc[c];
#pragma unroll
        for (int q = 0; q < kDin; q++) {
            const int e = threadIdx.x + q * kTriThreads;
            Dt[e / kTB][e % kTB] = dreg[q];
        }
        __syncthreads();
        // (2) reduced right-hand side of the block
#pragma unroll
        for (int q = 0; q < kRhs; q++) {
            const int e = threadIdx.x + q * kTriThreads;
            if (e < kTB * NB) {
                const int i = e % kTB, c = e / kTB;
                T sum = T(0);
#pragma unroll
                for (int ww = 0; ww < kTriWarps; ww++) sum += Red[(ww * NB + c) * kTB + i];
                Rb[i][c] = breg[q] - sum;
            }
        }
        __syncthreads();
        // (3) X_I = (L_II^-1)^T * Rb
        for (int e = threadIdx.x; e < kTB * NB; e += kTriThreads) {
            const int i = e % kTB, c = e / kTB;
            T x = T(0);
#pragma unroll 8
            for (int ip = 0; ip < kTB; ip++) x = fma(Dt[i][ip], Rb[ip][c], x);
            Xs[(r0 + i) * NB + c] = x;
            const int64_t gi = r0 + i, gc = c0 + c;
            if (gi < n && gc < n) Xout[gi * n + gc] = x;
        }
        __syncthreads();
        if (I > 0) {
#pragma unroll
            for (int q = 0; q < kDin; q++) dreg[q] = dnext[q];
#pragma unroll
            for (int q = 0; q < kRhs; q++) breg[q] = bnext[q];
        }
    }
    __pipeline_wait_prior(0);
}

// F = D_u A and H = T' D_xi A (column-major n x n): one warp per column b, a warp scan down the
// rows: H[c][b] = sum_{b <= k < c} xi_k A[k][b] + xi_c A[c][b] / 2 (zero above the diagonal).
template <typename T>
__global__ void k_pullback_fh(const T* __restrict__ A, const T* __restrict__ u,
                              const T* __restrict__ xi, int64_t n, T* __restrict__ F,
                              T* __restrict__ H) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t b = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < n;
         b += warps) {
        const T* a = A + b * n;
        T* f = F + b * n;
        T* h = H + b * n;
        T carry = T(0);
        for (int64_t c0 = 0; c0 < n; c0 += 32) {
            const int64_t c = c0 + lane;
            const bool in = c < n;
            const T av = (in && c >= b) ? a[c] : T(0);
            const T g = in ? xi[c] * av : T(0);
            T incl = g;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const T t = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += t;
            }
            if (in) {
                f[c] = u[c] * av;
                h[c] = carry + incl - T(0.5) * g;
            }
            carry += __shfl_sync(0xffffffffu, incl, 31);
        }
    }
}

template <typename T, int NB>
size_t trsm_smem(int64_t n) {
    const int64_t npad = (n + kTB - 1) / kTB * kTB;
    return sizeof(T) * ((size_t)tri_stages<T>() * kTileRows * kTB + (size_t)npad * NB +
                        (size_t)kTriWarps * kTB * NB + kTB * (NB + 1) + kTB * (kTB + 1));
}

constexpr size_t kTriSmemMax = 220 * 1024;

template <typename T, int NB>
int launch_trsm(gpb2_problem* p, bool gen, const T* u, const T* xi, const T* Bin, T* Xout,
                cudaStream_t s) {
    const int64_t n = p->n0;
    const size_t smem = trsm_smem<T, NB>(n);
    const unsigned grid = (unsigned)((n + NB - 1) / NB);
    const T* Lr = static_cast<const T*>(p->Ldr);
    const T* Di = static_cast<const T*>(p->Dinv);
    const int64_t ld = tri_pitch(n);
    if (gen) {
        GPB2_CUDA_TRY(prepare_kernel_smem((const void*)k_trsm_lt<T, NB, true>, smem));
        GPB2_CUDA_TRY(launch_prof("dense_trsm", k_trsm_lt<T, NB, true>, dim3(grid),
                                  dim3(kTriThreads), smem, s, Lr, ld, Di, u, xi,
                                  (const T*)nullptr, Xout, n));
    } else {
        GPB2_CUDA_TRY(prepare_kernel_smem((const void*)k_trsm_lt<T, NB, false>, smem));
        GPB2_CUDA_TRY(launch_prof("dense_trsm", k_trsm_lt<T, NB, false>, dim3(grid),
                                  dim3(kTriThreads), smem, s, Lr, ld, Di, (const T*)nullptr,
                                  (const T*)nullptr, Bin, Xout, n));
    }
    return GPB2_OK;
}

// Right-hand-side columns per CTA: about one CTA per SM, within the shared memory.
template <typename T>
int trsm_lt(gpb2_problem* p, bool gen, const T* u, const T* xi, const T* Bin, T* Xout,
            cudaStream_t s) {
    const int64_t n = p->n0;
    if (n > 8 * 148 && trsm_smem<T, 16>(n) <= kTriSmemMax)
        return launch_trsm<T, 16>(p, gen, u, xi, Bin, Xout, s);
    if (n > 4 * 148 && trsm_smem<T, 8>(n) <= kTriSmemMax)
        return launch_trsm<T, 8>(p, gen, u, xi, Bin, Xout, s);
    return launch_trsm<T, 4>(p, gen, u, xi, Bin, Xout, s);
}

inline cublasStatus_t gemm_sb(cublasHandle_t h, cublasOperation_t ta, cublasOperation_t tb,
                              int m, int nn, int k, float alpha, const float* A, int lda,
                              long long sA, const float* B, int ldb, long long sB, float beta,
                              float* C, int ldc, long long sC, int batch) {
    return cublasSgemmStridedBatched(h, ta, tb, m, nn, k, &alpha, A, lda, sA, B, ldb, sB, &beta,
                                     C, ldc, sC, batch);
}
inline cublasStatus_t gemm_sb(cublasHandle_t h, cublasOperation_t ta, cublasOperation_t tb,
                              int m, int nn, int k, double alpha, const double* A, int lda,
                              long long sA, const double* B, int ldb, long long sB, double beta,
                              double* C, int ldc, long long sC, int batch) {
    return cublasDgemmStridedBatched(h, ta, tb, m, nn, k, &alpha, A, lda, sA, B, ldb, sB, &beta,
                                     C, ldc, sC, batch);
}

#define GPB2_TRI_BLAS(expr)                                                                      \
    do {                                                                                         \
        cublasStatus_t _b = (expr);                                                              \
        if (_b != CUBLAS_STATUS_SUCCESS)                                                         \
            return set_error(GPB2_ERR_CUDA, "%s:%d: cuBLAS status %d", __FILE__, __LINE__,       \
                             (int)_b);                                                           \
    } while (0)

// A = L^-1 by recursive doubling (see the top of the file).  W: n*n/2 + n entries of work.
// The first doubling levels of L^-1 for one 128 x 128 diagonal block per CTA, in shared memory:
// from the inverted 32 x 32 diagonal blocks (Dinv), A21 = -A22 (L21 A11) for the 32- and then
// the 64-wide pairs, so the library GEMMs start at 128 (eight small launches fewer).  Not an
// exact-order computation: fused multiply-adds.
constexpr int kIB = 128;             // block of k_inv_block
constexpr int kIBP = kIB + 1;        // its row pitch in shared memory
constexpr int kIW = 64, kIWP = 65;   // the W scratch of one pair
template <typename T>
size_t inv_block_smem() { return sizeof(T) * ((size_t)kIB * kIBP + (size_t)kIW * kIWP); }

// out[r][c] = alpha * sum_k X[r][k] Y[k][c] for r < rows <= 64, c < cols <= 64 (row pitches
// given); each of 256 threads owns a 4 x 4 patch.
template <typename T>
__device__ __forceinline__ void cta_gemm64(T* out, int ldo, const T* X, int ldx, const T* Y,
                                           int ldy, int rows, int cols, int K, T alpha) {
    const int tr = (threadIdx.x >> 4) * 4, tc = (threadIdx.x & 15) * 4;
    if (tr >= rows || tc >= cols) return;
    T acc[4][4] = {};
#pragma unroll 8
    for (int k = 0; k < K; k++) {
        T xv[4], yv[4];
#pragma unroll
        for (int a = 0; a < 4; a++) xv[a] = tr + a < rows ? X[(tr + a) * ldx + k] : T(0);
#pragma unroll
        for (int b = 0; b < 4; b++) yv[b] = tc + b < cols ? Y[k * ldy + tc + b] : T(0);
#pragma unroll
        for (int a = 0; a < 4; a++)
#pragma unroll
            for (int b = 0; b < 4; b++) acc[a][b] = fma(xv[a], yv[b], acc[a][b]);
    }
#pragma unroll
    for (int a = 0; a < 4; a++)
#pragma unroll
        for (int b = 0; b < 4; b++)
            if (tr + a < rows && tc + b < cols) out[(tr + a) * ldo + tc + b] = alpha * acc[a][b];
}

template <typename T>
__global__ void __launch_bounds__(256) k_inv_block(const T* __restrict__ L,
                                                   const T* __restrict__ DinvT, int64_t n,
                                                   T* __restrict__ A) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T* M = reinterpret_cast<T*>(smem_raw);  // M[i * kIBP + j]: the block, row-major
    T* W = M + kIB * kIBP;
    const int64_t g0 = (int64_t)blockIdx.x * kIB;
    const int m = (int)(n - g0 < kIB ? n - g0 : kIB);
    // Staged in rounds of 16 elements per thread: all of a round's loads are issued before any
    // is stored (one memory latency per round, not per element).
    constexpr int kRound = 16;
    for (int e0 = 0; e0 < kIB * kIB; e0 += 256 * kRound) {
        T v[kRound];
#pragma unroll
        for (int u = 0; u < kRound; u++) {
            const int e = e0 + u * 256 + (int)threadIdx.x;
            const int i = e % kIB, j = e / kIB;  // coalesced along the column-major factor
            v[u] = T(0);
            if (i < m && j < m && i >= j) {
                if (i / kTB == j / kTB) {
                    const int64_t b = (g0 + i) / kTB;  // g0 is a multiple of kTB
                    v[u] = DinvT[b * kTB * kTB + (j % kTB) * kTB + (i % kTB)];
                } else {
                    v[u] = L[(g0 + i) + (g0 + j) * n];
                }
            }
        }
#pragma unroll
        for (int u = 0; u < kRound; u++) {
            const int e = e0 + u * 256 + (int)threadIdx.x;
            M[(e % kIB) * kIBP + e / kIB] = v[u];
        }
    }
    __syncthreads();
    for (int sz = kTB; sz < kIB; sz *= 2) {
        // W_p = L21 A11 for every pair p at this level, then A21 = -A22 W_p.
        for (int pass = 0; pass < 2; pass++) {
            for (int a0 = 0; a0 + sz < m; a0 += 2 * sz) {
                const int b0 = a0 + sz, s2 = m - b0 < sz ? m - b0 : sz;
                T* Wp = W + (a0 / (2 * sz)) * (sz == kTB ? kTB * kIWP : 0);
                if (pass == 0)
                    cta_gemm64(Wp, kIWP, M + b0 * kIBP + a0, kIBP, M + a0 * kIBP + a0, kIBP, s2,
                               sz, sz, T(1));
                else
                    cta_gemm64(M + b0 * kIBP + a0, kIBP, M + b0 * kIBP + b0, kIBP, Wp, kIWP, s2,
                               sz, s2, T(-1));
            }
            __syncthreads();
        }
    }
    for (int e = threadIdx.x; e < kIB * kIB; e += blockDim.x) {
        const int i = e % kIB, j = e / kIB;
        if (i < m && j < m) A[(g0 + i) + (g0 + j) * n] = M[i * kIBP + j];  // zeros above
    }
}

template <typename T>
int build_inverse(gpb2_problem* p, T* A, T* W, cudaStream_t s) {
    const int64_t n = p->n0;
    const T* L = static_cast<const T*>(p->Ld);
    // A's upper triangle is zero from its allocation and nothing writes there: k_inv_block
    // writes the whole 128-wide diagonal blocks (zeros above their diagonal included) and the
    // GEMMs below write only blocks below the diagonal.  Levels 32 and 64 inside each
    // 128-wide diagonal block, then library GEMMs from 128 up.
    const size_t ism = inv_block_smem<T>();
    GPB2_CUDA_TRY(prepare_kernel_smem((const void*)k_inv_block<T>, ism));
    GPB2_CUDA_TRY(launch_prof("dense_inv_block", k_inv_block<T>,
                              dim3((unsigned)((n + kIB - 1) / kIB)), dim3(256), ism, s, L,
                              (const T*)p->Dinv, n, A));
    GPB2_TRI_BLAS(cublasSetStream(p->blas, s));
    const int ni = (int)n;
    for (int64_t sz = kIB; sz < n; sz *= 2) {
        const int64_t full = n / (2 * sz);  // complete pairs (A11, A22 both of size sz)
        const long long diag = 2 * sz * (n + 1);  // stride between pairs along the diagonal
        const int si = (int)sz;
        if (full > 0) {
            // W_b = L21 A11, then A21 = -A22 W_b
            GPB2_TRI_BLAS(gemm_sb(p->blas, CUBLAS_OP_N, CUBLAS_OP_N, si, si, si, T(1), L + sz, ni,
                                  diag, A, ni, diag, T(0), W, si, (long long)sz * sz,
                                  (int)full));
            GPB2_TRI_BLAS(gemm_sb(p->blas, CUBLAS_OP_N, CUBLAS_OP_N, si, si, si, T(-1),
                                  A + sz * (n + 1), ni, diag, W, si, (long long)sz * sz, T(0),
                                  A + sz, ni, diag, (int)full));
        }
        const int64_t j = full * 2 * sz;  // a trailing A11 of size sz with a shorter A22
        const int64_t r = n - j - sz;
        if (r > 0) {
            const int ri = (int)r;
            GPB2_TRI_BLAS(gemm_sb(p->blas, CUBLAS_OP_N, CUBLAS_OP_N, ri, si, si, T(1),
                                  L + (j + sz) + j * n, ni, 0, A + j + j * n, ni, 0, T(0), W, ri,
                                  0, 1));
            GPB2_TRI_BLAS(gemm_sb(p->blas, CUBLAS_OP_N, CUBLAS_OP_N, ri, si, ri, T(-1),
                                  A + (j + sz) + (j + sz) * n, ni, 0, W, ri, 0, T(0),
                                  A + (j + sz) + j * n, ni, 0, 1));
        }
    }
    return GPB2_OK;
}

}  // namespace

template <typename T>
bool dense_tri_supported(const gpb2_problem* p) {
    return trsm_smem<T, 4>(p->n0) <= kTriSmemMax;
}

template <typename T>
int dense_tri_prepare(gpb2_problem* p, cudaStream_t s, cudaEvent_t after_ldr) {
    const int64_t n = p->n0, ld = tri_pitch(n);
    const int64_t nbk = (n + kTB - 1) / kTB;
    const size_t nn = (size_t)n * (size_t)n;
    GPB2_TRY(ensure_alloc(&p->Ldr, sizeof(T) * (size_t)n * (size_t)ld));
    GPB2_TRY(ensure_alloc(&p->Dinv, sizeof(T) * (size_t)nbk * kTB * kTB));
    GPB2_TRY(ensure_alloc(&p->Wtri, sizeof(T) * (2 * nn + (size_t)n)));
    if (!p->Ainv) {
        GPB2_TRY(ensure_alloc(&p->Ainv, sizeof(T) * nn));
        GPB2_CUDA_TRY(cudaMemsetAsync(p->Ainv, 0, sizeof(T) * nn, s));  // upper triangle: zero
    }
    GPB2_CUDA_TRY(launch_prof("dense_transpose", k_transpose_lower<T>,
                              dim3((unsigned)std::min<int64_t>(nbk * nbk, 4 * 148)),
                              dim3(kTriThreads), 0, s, (const T*)p->Ld, (T*)p->Ldr, n, ld));
    if (after_ldr) GPB2_CUDA_TRY(cudaEventRecord(after_ldr, s));
    GPB2_CUDA_TRY(launch_prof("dense_diag_inv", k_diag_inv<T>,
                              dim3((unsigned)((nbk + kDiagWarps - 1) / kDiagWarps)),
                              dim3(32 * kDiagWarps), 0, s, (const T*)p->Ldr, n, ld,
                              (T*)p->Dinv));
    const ProfToken t = prof_begin("dense_inverse", s);
    const int st = build_inverse<T>(p, static_cast<T*>(p->Ainv), static_cast<T*>(p->Wtri), s);
    prof_end(t, s);
    return st;
}

template <typename T>
int dense_trmv(gpb2_problem* p, bool trans, const T* x, T* y, cudaStream_t s) {
    const int64_t n = p->n0;
    const dim3 grid((unsigned)((n + 31) / 32));
    if (trans)
        GPB2_CUDA_TRY(launch_prof("dense_trmv", k_trmv_exact<T, true>, grid, dim3(kTrmvThreads),
                                  0, s, (const T*)p->Ldr, tri_pitch(n), x, y, n));
    else
        GPB2_CUDA_TRY(launch_prof("dense_trmv", k_trmv_exact<T, false>, grid, dim3(kTrmvThreads),
                                  0, s, (const T*)p->Ld, n, x, y, n));
    return GPB2_OK;
}

template <typename T>
int dense_chol_pullback_outer(gpb2_problem* p, const T* vb, const T* xi, const T** S_out,
                              cudaStream_t s) {
    const int64_t n = p->n0;
    const size_t nn = (size_t)n * (size_t)n;
    T* F = static_cast<T*>(p->Wtri);
    T* H = F + nn;
    T* u = H + nn;
    T* S = static_cast<T*>(p->Wd2);
    GPB2_TRY(dense_trmv<T>(p, true, vb, u, s));  // u = L^T vb
    GPB2_CUDA_TRY(launch_prof("dense_pullback_fh", k_pullback_fh<T>,
                              dim3((unsigned)std::min<int64_t>((n + 7) / 8, 8 * 148)),
                              dim3(256), 0, s, (const T*)p->Ainv, (const T*)u, xi, n, F, H));
    GPB2_TRI_BLAS(cublasSetStream(p->blas, s));
    const int ni = (int)n;
    const ProfToken t = prof_begin("dense_gemm", s);
    const cublasStatus_t st = gemm_sb(p->blas, CUBLAS_OP_T, CUBLAS_OP_N, ni, ni, ni, T(1), F, ni,
                                      0, H, ni, 0, T(0), S, ni, 0, 1);  // S = F^T H
    prof_end(t, s);
    GPB2_TRI_BLAS(st);
    *S_out = S;  // column-major S
    return GPB2_OK;
}

template bool dense_tri_supported<float>(const gpb2_problem*);
template bool dense_tri_supported<double>(const gpb2_problem*);
template int dense_tri_prepare<float>(gpb2_problem*, cudaStream_t, cudaEvent_t);
template int dense_tri_prepare<double>(gpb2_problem*, cudaStream_t, cudaEvent_t);
template int dense_trmv<float>(gpb2_problem*, bool, const float*, float*, cudaStream_t);
template int dense_trmv<double>(gpb2_problem*, bool, const double*, double*, cudaStream_t);
template int dense_chol_pullback_outer<float>(gpb2_problem*, const float*, const float*,
                                              const float**, cudaStream_t);
template int dense_chol_pullback_outer<double>(gpb2_problem*, const double*, const double*,
                                               const double**, cudaStream_t);

}  // namespace gpb2
