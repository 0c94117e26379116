// Quantized mul_mat with 9 or more activation rows (prefill) on the 5th-generation tensor cores.
//
// out[m][n] = sum over blocks b, in order, of fma(d_w[n][b] * d_x[m][b], isum(n, m, b), .), the
// order the CPU checker uses for this many rows. isum is the exact integer dot product of a weight
// block (Q4_0 codes - 8, or Q8_0 codes) with the Q8_0-quantized activation block: one
// tcgen05.mma.kind::i8 (M = 128 weight rows, N = 64 activation rows, K = 32 = one block) per block
// computes it for a whole tile into tensor memory, exactly; the fp32 scaling chain runs on the
// CUDA cores in block order.
//
// CTA: warps 0-15 epilogue (warp w reads TMEM lanes 32*(w%4).., columns 16*(w/4)..), warps 16-19
// loaders, warp 20 the MMA issuer (one thread) and TMEM owner. A stage holds KB = 4 blocks: the
// tile's weight blocks (128 x 32 int8 each) and activation blocks (64 x 32 int8 each) in the
// no-swizzle K-major UMMA layout plus their scales, and 4 x 64 TMEM columns for the MMA results. Loaders bring raw
// blocks in 8-block chunks with cp.async, three chunks ahead. Barriers: full (loaders -> MMA), done
// (MMA -> epilogue, via tcgen05.commit), free (epilogue -> loaders and MMA). Every wait is bounded
// in time; a timeout sets the error word (2), turns the rest of the CTA's work off and lets it
// release its tensor memory.
#include <cuda_fp16.h>

#include <stdexcept>
#include <string>

#include "../gc_kernels.h"
#include "gc_math.cuh"
#include "gc_qweight.cuh"
#include "gc_tma.cuh"

namespace gcb {
namespace k {

namespace {

constexpr int BM = 128;          // weight rows per tile (UMMA M)
constexpr int BN = 64;           // activation rows per tile (UMMA N)
constexpr int KB = 4;            // blocks per stage (one barrier round trip per KB blocks)
constexpr int S = 2;             // stages
constexpr int CK = 8;            // blocks per raw chunk
constexpr int RB = 3;            // raw chunk buffers
constexpr int NEPI = 16, NLD = 4; // epilogue and loader warps
constexpr int EC = BN / (NEPI / 4);  // activation columns per epilogue warp
constexpr int NTHREADS = (NEPI + NLD + 1) * 32;
constexpr int TMEM_COLS = S * KB * BN;  // 512: the whole tensor memory of the SM (one CTA per SM)

constexpr int A_BYTES = BM * 32, B_BYTES = BN * 32;  // one block
constexpr int A_LBO = BM * 16, B_LBO = BN * 16;  // bytes between the two 16-byte K halves

struct GemmArgs {
    const char *w;        // tiled weight (gc_qweight.cuh)
    int nb, cb;           // blocks per row, code bytes per block
    int N, M;             // weight rows, activation rows
    const int8_t *qx;     // activation codes [M][K]
    const uint16_t *dx;   // activation scales [M][nb] (fp16)
    float *out;           // [M][N]
    int *err;
};

// UMMA shared-memory descriptor: no swizzle, K-major (8-row core matrices of 16 bytes).
__device__ __forceinline__ uint64_t smem_desc(const void *p, uint32_t lbo, uint32_t sbo) {
    const uint32_t a = smem_u32(p);
    return (uint64_t)((a >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46);  // version 1, base offset 0, layout 0
}

// Instruction descriptor: D s32, A s8, B s8, both K-major, N = BN, M = BM.
constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Packed f32x2 arithmetic (sm_100): two independent IEEE single-precision operations, low word
// first; the results are those of the scalar operations.
__device__ __forceinline__ uint64_t f2pack(float lo, float hi) {
    return ((uint64_t)__float_as_uint(hi) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ uint64_t f32x2_mul(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f32x2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f32x2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
constexpr uint64_t kBias2 = 0xCB400000CB400000ull;  // (-12582912.0f, -12582912.0f)

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

// Waits for this thread's outstanding tensor-memory loads; `r` (the registers of the last load) pass
// through the wait, so the compiler cannot move their uses above it.
__device__ __forceinline__ void tmem_wait(uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
                 :
                 : "memory");
}

// The low nibbles of four bytes as signed bytes (q - 8): q + 0x78 stays below 0x100 (no carry into
// the next byte) and flipping its top bit subtracts 0x80.
__device__ __forceinline__ uint32_t q4_lo(uint32_t w) { return ((w & 0x0f0f0f0fu) + 0x78787878u) ^ 0x80808080u; }

// Bounded wait shared by the CTA: once one wait has timed out every later wait returns false.
__device__ __forceinline__ bool wait_ok(uint64_t *bar, uint32_t parity, volatile int *abort, int *err) {
    if (*abort) return false;
    if (mbar_wait_sleep(bar, parity)) return true;
    *abort = 1;
    if (err) atomicExch(err, 2);
    return false;
}

// The same, uniform across the warp: lane 0 waits and shares the outcome (the warp then runs
// warp-collective instructions together).
__device__ __forceinline__ bool warp_wait_ok(uint64_t *bar, uint32_t parity, volatile int *abort, int *err) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0) ok = wait_ok(bar, parity, abort, err) ? 1 : 0;
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

template <int QT>
__global__ void __launch_bounds__(NTHREADS, 1) gemm_tc_kernel(GemmArgs g) {
    constexpr int CB = QT == 0 ? 16 : 32;
    extern __shared__ __align__(1024) unsigned char smem[];
    // stages
    unsigned char *As = smem;                                  // [S][KB][A_BYTES]
    unsigned char *Bs = As + S * KB * A_BYTES;                 // [S][KB][B_BYTES]
    float *dws = (float *)(Bs + S * KB * B_BYTES);             // [S][KB][BM]
    float *dxs = dws + S * KB * BM;                            // [S][KB][BN]
    // raw chunks: block-major so a thread's reads of one block are contiguous across threads
    unsigned char *Araw = (unsigned char *)(dxs + S * KB * BN);  // [RB][CK][BM][CB]
    uint16_t *Ascl = (uint16_t *)(Araw + RB * CK * BM * CB);   // [RB][BM][CK]
    unsigned char *Braw = (unsigned char *)(Ascl + RB * BM * CK);  // [RB][CK][BN][32]
    uint16_t *Bscl = (uint16_t *)(Braw + RB * CK * BN * 32);   // [RB][BN][CK]
    __shared__ __align__(8) uint64_t full[S], done[S], freeb[S];
    __shared__ uint32_t tmem_base;
    __shared__ int s_abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BM, m0 = blockIdx.y * BN;
    const int nb = g.nb;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], NLD);
            mbar_init(&done[s], 1);
            mbar_init(&freeb[s], NEPI);
        }
        mbar_fence_init();
        s_abort = 0;
    }
    if (warp == NEPI + NLD) {  // the MMA warp owns the tensor memory
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = tmem_base;

    if (warp < NEPI) {
        // ------------------------------------------------------------ epilogue
        const int q = warp & 3, h = warp >> 2;
        const int row = q * 32 + lane;  // weight row within the tile = TMEM lane
        uint64_t acc2[EC / 2];  // two f32 sums per register pair
#pragma unroll
        for (int i = 0; i < EC / 2; i++) acc2[i] = 0ull;
        const int nst = nb / KB;
        for (int st = 0; st < nst; st++) {
            const int s = st % S;
            // full: this stage's scales (plain stores by the loaders) are visible; done: its MMAs are complete
            if (!warp_wait_ok(&full[s], (uint32_t)((st / S) & 1), &s_abort, g.err)) break;
            if (!warp_wait_ok(&done[s], (uint32_t)((st / S) & 1), &s_abort, g.err)) break;
            tc_fence_after();
            const uint32_t t0 = tbase + ((uint32_t)(q * 32) << 16) + (uint32_t)(s * KB * BN + h * EC);
            uint32_t v[2][EC];
            tmem_ld16(t0, v[0]);
            tmem_wait(v[0]);
#pragma unroll
            for (int j = 0; j < KB; j++) {  // blocks in order; the next block's TMEM load overlaps this one's math
                if (j + 1 < KB) tmem_ld16(t0 + (uint32_t)((j + 1) * BN), v[(j + 1) & 1]);
                const float dw = dws[(s * KB + j) * BM + row];
                const float *dxr = dxs + (s * KB + j) * BN + h * EC;
                const uint64_t dw2 = f2pack(dw, dw);
#pragma unroll
                for (int c = 0; c < EC; c += 2) {
                    // acc = fma(dw * dx, (float)isum, acc) for two columns at once (packed f32x2,
                    // each lane an ordinary IEEE op); isum -> float exactly through the 1.5 * 2^23
                    // bias (|isum| <= 32 * 127 * 127 < 2^22)
                    const uint64_t p2 = f32x2_mul(dw2, *(const uint64_t *)(dxr + c));
                    const uint64_t i2 = f2pack(__uint_as_float(v[j & 1][c] + 0x4B400000u), __uint_as_float(v[j & 1][c + 1] + 0x4B400000u));
                    acc2[c / 2] = f32x2_fma(p2, f32x2_add(i2, kBias2), acc2[c / 2]);
                }
                if (j + 1 < KB) tmem_wait(v[(j + 1) & 1]);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&freeb[s]);
        }
        const int n = n0 + row;
        if (n < g.N && !s_abort)
#pragma unroll
            for (int i = 0; i < EC; i++) {
                const int m = m0 + h * EC + i;
                if (m < g.M) g.out[(int64_t)m * g.N + n] = __uint_as_float((unsigned)(acc2[i / 2] >> (32 * (i & 1))));
            }
    } else if (warp < NEPI + NLD) {
        // ------------------------------------------------------------ loaders
        const int t = threadIdx.x - NEPI * 32;  // 0..127: weight row t; activation row t (t < 64)
        const int n = n0 + t;
        const int xr = t >> 1, hb = t & 1;  // activation row and K half of this thread
        const int npad = (g.N + QTR - 1) / QTR * QTR;
        const bool wrow = n < npad, xrow = m0 + xr < g.M;
        const int nchunks = nb / CK;
        auto issue = [&](int c) {
            const int rb = c % RB, kb0 = c * CK;
            if (wrow) {
                const int64_t seg = kb0 / QSEG, sb = qw_seg_blocks(nb, seg);
                const unsigned char *piece = (const unsigned char *)g.w + qw_piece_off(nb, CB, n / QTR, seg);
                const unsigned char *codes = piece + ((n % QTR) * sb + kb0 % QSEG) * CB;
                const unsigned char *scl = piece + QTR * sb * CB + ((n % QTR) * sb + kb0 % QSEG) * 2;
#pragma unroll
                for (int j = 0; j < CK; j++)
#pragma unroll
                    for (int e = 0; e < CB; e += 16) cp_async16(Araw + ((rb * CK + j) * BM + t) * CB + e, codes + j * CB + e);
                cp_async16(Ascl + (rb * BM + t) * CK, scl);
            }
            if (xrow) {  // K half hb of activation row xr
                const int8_t *xs = g.qx + (int64_t)(m0 + xr) * nb * 32 + (int64_t)kb0 * 32 + hb * 16;
#pragma unroll
                for (int j = 0; j < CK; j++) cp_async16(Braw + ((rb * CK + j) * BN + xr) * 32 + hb * 16, xs + j * 32);
                if (hb == 0) cp_async16(Bscl + (rb * BN + xr) * CK, g.dx + (int64_t)(m0 + xr) * nb + kb0);
            }
            cp_async_commit();
        };
        for (int c = 0; c < RB - 1; c++) {
            if (c < nchunks) issue(c);
            else cp_async_commit();
        }
        for (int c = 0; c < nchunks; c++) {
            if (c + RB - 1 < nchunks) issue(c + RB - 1);
            else cp_async_commit();
            cp_async_wait<RB - 1>();  // this thread's copies of chunk c have landed
            const int rb = c % RB;
            bool ok = true;
            for (int j0 = 0; j0 < CK; j0 += KB) {  // the chunk's stages
                const int st = (c * CK + j0) / KB, s = st % S;
                if (st >= S && !warp_wait_ok(&freeb[s], (uint32_t)(((st / S) - 1) & 1), &s_abort, g.err)) {
                    ok = false;
                    break;
                }
                // every shared-memory load of the stage first
                uint4 craw[KB][CB / 16], braw[KB];
                uint16_t wsc[KB], xsc[KB];
#pragma unroll
                for (int jj = 0; jj < KB; jj++) {
                    const unsigned char *src = Araw + ((rb * CK + j0 + jj) * BM + t) * CB;
#pragma unroll
                    for (int e = 0; e < CB / 16; e++) craw[jj][e] = wrow ? *(const uint4 *)(src + e * 16) : make_uint4(0, 0, 0, 0);
                    wsc[jj] = wrow ? Ascl[(rb * BM + t) * CK + j0 + jj] : (uint16_t)0;
                    braw[jj] = xrow ? *(const uint4 *)(Braw + ((rb * CK + j0 + jj) * BN + xr) * 32 + hb * 16) : make_uint4(0, 0, 0, 0);
                    xsc[jj] = xrow ? Bscl[(rb * BN + xr) * CK + j0 + jj] : (uint16_t)0;
                }
                // weight blocks of row t -> int8 in the UMMA layout (two 16-byte K halves); activation
                // row xr, K half hb
#pragma unroll
                for (int jj = 0; jj < KB; jj++) {
                    uint4 lo, hi;
                    if (QT == 0) {
                        const uint4 c4 = craw[jj][0];
                        lo = make_uint4(q4_lo(c4.x), q4_lo(c4.y), q4_lo(c4.z), q4_lo(c4.w));
                        hi = make_uint4(q4_lo(c4.x >> 4), q4_lo(c4.y >> 4), q4_lo(c4.z >> 4), q4_lo(c4.w >> 4));
                        if (!wrow) lo = hi = make_uint4(0, 0, 0, 0);
                    } else {
                        lo = craw[jj][0];
                        hi = craw[jj][CB / 16 - 1];
                    }
                    unsigned char *a = As + (s * KB + jj) * A_BYTES + (t >> 3) * 128 + (t & 7) * 16;
                    *(uint4 *)a = lo;
                    *(uint4 *)(a + A_LBO) = hi;
                    dws[(s * KB + jj) * BM + t] = wrow ? h2f(wsc[jj]) : 0.0f;
                    *(uint4 *)(Bs + (s * KB + jj) * B_BYTES + hb * B_LBO + (xr >> 3) * 128 + (xr & 7) * 16) = braw[jj];
                    if (hb == 0) dxs[(s * KB + jj) * BN + xr] = xrow ? h2f(xsc[jj]) : 0.0f;
                }
                fence_proxy_async_shared();  // the generic stores above are visible to the tensor core
                __syncwarp();
                if (lane == 0) mbar_arrive(&full[s]);
            }
            if (!ok) break;
        }
        cp_async_wait<0>();
    } else if (lane == 0) {
        // ------------------------------------------------------------ MMA issuer
        int last = -1;
        for (int st = 0; st < nb / KB; st++) {
            const int s = st % S;
            if (!wait_ok(&full[s], (uint32_t)((st / S) & 1), &s_abort, g.err)) break;
            tc_fence_after();
#pragma unroll
            for (int j = 0; j < KB; j++) {  // one MMA per block, each into its own TMEM columns
                const uint64_t ad = smem_desc(As + (s * KB + j) * A_BYTES, A_LBO, 128);
                const uint64_t bd = smem_desc(Bs + (s * KB + j) * B_BYTES, B_LBO, 128);
                const uint32_t d = tbase + (uint32_t)((s * KB + j) * BN);
                asm volatile(
                    "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                    "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
                    "l"(ad), "l"(bd), "r"(IDESC), "r"(0));
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             smem_u32(&done[s]))
                         : "memory");
            last = st;
        }
        if (last >= 0) mbar_wait(&done[last % S], (uint32_t)((last / S) & 1), 100000000ull);  // the last MMAs are complete
    }

    tc_fence_before();
    __syncthreads();
    if (warp == NEPI + NLD) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(TMEM_COLS));
    }
}

size_t smem_bytes(int cb) {
    return (size_t)S * KB * (A_BYTES + B_BYTES) + (size_t)S * KB * (BM + BN) * 4 + (size_t)RB * CK * BM * cb + (size_t)RB * BM * CK * 2 +
           (size_t)RB * CK * BN * 32 + (size_t)RB * BN * CK * 2;
}

}  // namespace

bool gemm_tc_ok(const TD &a, const TD &b) {
    if (a.type != T_Q4_0 && a.type != T_Q8_0) return false;
    if (a.ne[2] != 1 || a.ne[3] != 1 || b.ne[2] != 1 || b.ne[3] != 1 || b.ne[1] < GEMM_MIN_ROWS) return false;
    return (a.ne[0] / 32) % CK == 0 && CK % KB == 0 && a.ne[1] < (1 << 30) && b.ne[1] < (1 << 30);
}

void gemm_tc(const TD &a, int64_t M, const int8_t *qx, const uint16_t *dx, float *out, int *err, cudaStream_t s) {
    GemmArgs g;
    g.w = a.data;
    g.nb = (int)(a.ne[0] / 32);
    g.cb = a.type == T_Q4_0 ? 16 : 32;
    g.N = (int)a.ne[1];
    g.M = (int)M;
    g.qx = qx;
    g.dx = dx;
    g.out = out;
    g.err = err;
    const size_t smem = smem_bytes(g.cb);
    auto kern = a.type == T_Q4_0 ? gemm_tc_kernel<0> : gemm_tc_kernel<1>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const dim3 grid((unsigned)((g.N + BM - 1) / BM), (unsigned)((g.M + BN - 1) / BN));
    kern<<<grid, NTHREADS, smem, s>>>(g);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) throw std::runtime_error(std::string("CUDA launch of gemm_tc failed: ") + cudaGetErrorString(e));
}

}  // namespace k
}  // namespace gcb
