// Quantized GEMV for 2-8 activation rows (batched decode) with the block dot products on the tensor
// cores, each row's arithmetic still the one-row GEMV's (gc_gemv_dev.cuh), bit for bit.
//
// The one-row order per (weight row, activation row): block b's exact integer dot goes into chain
// b mod 32 as fma(d_w * d_x, dot, chain), blocks in increasing order, then the 32 chains are summed
// by the butterfly's pairs (chain k + chain k + 16, then + 8, 4, 2, 1). On CUDA cores every
// (weight row, activation row, block) costs 8 dp4a; here one mma.sync.m16n8k32 (int8, exact int32
// sums) gives a block's dots for 8 activation rows x 8 weight rows at once, and each thread keeps,
// for its (activation row m, weight rows n, n + 1) pair, the chains its warp owns:
//   - a team of 4 warps takes one 8-row tile piece at a time; warp q handles the blocks b with
//     b mod 32 in [8q, 8q + 8) (chains 8q .. 8q + 7), in increasing b;
//   - the MMA's A operand is the activation block (rows m; rows past M are read from row 0 and
//     their results dropped), B the 8 weight rows' block (Q4_0: the nibbles as unsigned bytes, with
//     8 x the activation code sum subtracted from the dot: the (q - 8) of Q4_0); thread (g, t) of
//     the warp gets C[g][2t], C[g][2t + 1]: activation row g, weight rows 2t and 2t + 1;
//   - at the end of a tile the four warps' chains meet through shared memory along the butterfly's
//     pairs (levels 16 and 8 across warps, 4, 2, 1 in warp 0), so the sum is the butterfly's value.
// Operands come through ldmatrix from shared memory laid out without bank conflicts: the producer
// copies each piece's 8 code rows with a 16-byte pad between them (9 bulk copies per piece), and
// the staged activation rows are K + 16 bytes apart.
//
// Persistent CTAs, one per SM: warp 8's lane 0 streams pieces into a ring (bounded waits, as in
// gc_fused.cu); warps 0-7 are two teams taking the CTA's row groups in chunks of two, segment-major
// inside a chunk. The activation rows come staged (FusedArgs::PRO_Q8, written by act_rows).
#include <cuda_fp16.h>

#include <cstdlib>
#include <stdexcept>
#include <string>

#include "gc_gemv_dev.cuh"

namespace gcb {
namespace k {

namespace {

constexpr int MMW = 8;                   // consumer warps
constexpr int MM_THREADS = (MMW + 1) * 32;
constexpr int MM_WPP = 4;                // warps per team (per piece)
constexpr int MM_TEAMS = MMW / MM_WPP;   // 2
constexpr int MM_MAXNS = 16;
constexpr int MM_MAXNR = 2;

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void *addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(addr)));
}

// C[g][2t], C[g][2t + 1] of one m16n8k32 integer MMA (rows g + 8 of A are zero: their results are
// not used). QT 0: B unsigned (Q4_0 nibbles), 1: signed (Q8_0 codes).
template <int QT>
__device__ __forceinline__ void mma_dot(int &c0, int &c1, uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
    int d2, d3;
    if constexpr (QT == 0)
        asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
                     "{%10, %10, %10, %10};"
                     : "=r"(c0), "=r"(c1), "=r"(d2), "=r"(d3)
                     : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1), "r"(0));
    else
        asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
                     "{%10, %10, %10, %10};"
                     : "=r"(c0), "=r"(c1), "=r"(d2), "=r"(d3)
                     : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1), "r"(0));
}

// Geometry of a slot: the piece's 8 code rows `rs` bytes apart (sb * CB + 16), then its 8 scale rows
// `ss` bytes apart (sb * 2 + 16): every row one bulk copy, each 16-byte pad moving the next row
// to other banks.
__host__ __device__ inline int mm_row_stride(int sb, int cb) { return sb * cb + 16; }
__host__ __device__ inline int mm_scale_stride(int sb) { return sb * 2 + 16; }
__host__ __device__ inline int mm_slot_bytes(int sb, int cb) { return QTR * (mm_row_stride(sb, cb) + mm_scale_stride(sb)); }
// Staged activation rows: scales (f16 bits) nb + 8 apart, code sums nb + 4 apart (16-byte pads).
__host__ __device__ inline int mm_dh_stride(int nb) { return nb + 8; }
__host__ __device__ inline int mm_s8_stride(int nb) { return nb + 4; }

// One row's epilogue value(s) y[r] for (activation row m, weight row `row` of matrix `mat`):
// the one-row GEMV's epilogue (gemv_epi_store) for one activation row.
template <int NR>
__device__ __forceinline__ void mm_epi(const FusedArgs &a, int mat, int row, int m, const float (&y)[NR], float e0, float e1) {
    if (a.map == MAP_SINGLE) {
        if (row >= a.wrows[0]) return;
        float v = y[0];
        if (a.res) v = __fadd_rn(e0, v);
        a.out[m * a.ldo + row] = v;
    } else if (a.map == MAP_SWIGLU) {
        if (row >= a.wrows[0]) return;
        a.out[m * a.ldo + row] = __fmul_rn(gc_silu(y[0]), y[NR - 1]);
    } else {
        const int D = (int)a.D, half = D / 2, h = row / D, i = row - h * D;
        const int32_t p = a.pos[m];
        float y0 = y[0], y1 = y[NR - 1];
        if (mat < 2) {
            float c, sn;
            if (p >= 0 && p < a.npos) {
                c = e0;
                sn = e1;
            } else {
                float theta = (float)p;
                for (int kk = 0; kk < i; kk++) theta = __fmul_rn(theta, a.theta_scale);
                c = cosf(theta);
                sn = sinf(theta);
            }
            const float x0 = y0, x1 = y1;
            y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
            y1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
        }
        if (mat == 0) {
            float *qo = a.q_out + m * a.ldq + (int64_t)h * D;
            qo[i] = y0;
            qo[i + half] = y1;
        } else if (p >= 0 && p < a.cache_rows) {
            char *base = (mat == 1 ? a.kcache : a.vcache) + m * a.cache_nb3 + p * a.cache_nb1 + h * a.cache_nb2;
            ((__half *)base)[i] = __float2half_rn(y0);
            ((__half *)base)[i + half] = __float2half_rn(y1);
        } else if (a.err) {
            atomicExch(a.err, 1);
        }
    }
}

// The epilogue operands of (m, row) loaded at a tile's start: residual, or RoPE cos / sin.
__device__ __forceinline__ void mm_epi_load(const FusedArgs &a, int mat, int row, int m, float &e0, float &e1) {
    e0 = e1 = 0.0f;
    if (a.map == MAP_SINGLE) {
        if (a.res && row < a.wrows[0]) e0 = a.res[m * a.ldr + row];
    } else if (a.map == MAP_ROPE_QKV && mat < 2) {
        const int D = (int)a.D, half = D / 2, i = row % D;
        const int32_t p = a.pos[m];
        if (p >= 0 && p < a.npos) {
            e0 = a.table[((int64_t)p * half + i) * 2];
            e1 = a.table[((int64_t)p * half + i) * 2 + 1];
        }
    }
}

template <int QT, int NR>
__global__ void __launch_bounds__(MM_THREADS, 1) gemv_mma_kernel(FusedArgs a, GemvGeo G, int ns, uint32_t magic, int slot_bytes) {
    extern __shared__ __align__(128) unsigned char smem[];
    constexpr int CB = QT == 0 ? 16 : 32;
    uint64_t *full = (uint64_t *)smem;
    uint64_t *empty = full + MM_MAXNS;
    float2 *xch = (float2 *)(empty + MM_MAXNS);  // [team][2][NR][8 chains][32 lanes] chain exchange
    const int K = (int)a.K, nb = G.nb, M = a.M, kp = K + 16;
    const int dhs = mm_dh_stride(nb), s8s = mm_s8_stride(nb);
    int8_t *sx = (int8_t *)(xch + MM_TEAMS * 2 * MM_MAXNR * 8 * 32);
    uint16_t *sdh = (uint16_t *)(sx + (size_t)M * kp);
    int *ss8 = (int *)(sdh + (size_t)M * dhs);  // nb + 8 halves a row: 16-byte aligned
    unsigned char *slots = (unsigned char *)smem + ((((size_t)((char *)(ss8 + (size_t)M * s8s) - (char *)smem)) + 127) & ~(size_t)127);
    const Ring R{full, empty, slots, (uint32_t)ns, magic, slot_bytes};
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < ns; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], MM_WPP);
        }
        mbar_fence_init();
    }
    __syncthreads();
    pdl_trigger();

    const int L = local_groups(G.groups, blockIdx.x, gridDim.x);
    const int per_group = G.nseg * G.pieces;

    if (warp == MMW) {  // producer: pieces in the consumers' order, each as 8 padded code rows + scales
        if (lane != 0) return;
        if (a.trace) a.trace[blockIdx.x * 8 + 0] = global_ns();
        const uint64_t policy = a.stream_evict_first ? l2_policy_evict_first() : 0;
        uint32_t t = 0;
        bool ok = true;
        for (int c0 = 0; c0 < L && ok; c0 += MM_TEAMS) {
            const int n = c0 + MM_TEAMS < L ? MM_TEAMS : L - c0;
            for (int s = 0; s < G.nseg && ok; s++) {
                const int sb = (int)qw_seg_blocks(nb, s), rs = mm_row_stride(sb, CB);
                for (int q = 0; q < n && ok; q++)
                    for (int r = 0; r < G.pieces; r++, t++) {
                        const int slot = R.slot(t);
                        if (t >= R.ns && !mbar_wait(&R.empty[slot], R.parity(t) ^ 1u)) {
                            ok = false;
                            break;
                        }
                        const uint32_t code_row = (uint32_t)(sb * CB), scl_row = (uint32_t)(sb * 2);
                        const int ss = mm_scale_stride(sb);
                        mbar_expect_tx(&R.full[slot], QTR * (code_row + scl_row));
                        int mat, tile;
                        const char *src = gemv_piece(a, G, (int)blockIdx.x + (c0 + q) * (int)gridDim.x, r, s, &mat, &tile);
                        unsigned char *dst = R.data(t);
                        for (int rr = 0; rr < QTR; rr++) {
                            unsigned char *dc = dst + rr * rs, *ds = dst + QTR * rs + rr * ss;
                            const char *sc = src + rr * code_row, *sl = src + QTR * code_row + rr * scl_row;
                            if (a.stream_evict_first) {
                                bulk_g2s_hint(dc, sc, code_row, &R.full[slot], policy);
                                bulk_g2s_hint(ds, sl, scl_row, &R.full[slot], policy);
                            } else {
                                bulk_g2s(dc, sc, code_row, &R.full[slot]);
                                bulk_g2s(ds, sl, scl_row, &R.full[slot]);
                            }
                        }
                    }
            }
        }
        if (!ok) {
            if (a.err) atomicExch(a.err, 2);
            drain_ring(R, t);
        } else if (a.trace) {
            a.trace[blockIdx.x * 8 + 1] = global_ns();
        }
        return;
    }

    pdl_wait();  // the staged rows were written by the kernel before
    const bool stamp = a.trace && threadIdx.x == 0;
    if (stamp) a.trace[blockIdx.x * 8 + 2] = global_ns();
    {  // staged rows -> shared memory: codes with the row pad, scales as f16 bits, code sums
        const int8_t *gc = (const int8_t *)a.xq;
        const float *gd = (const float *)(a.xq + (size_t)M * K);
        const int *gs = (const int *)(gd + (size_t)M * nb);
        const int n16 = K / 16;
        for (int i = threadIdx.x; i < M * n16; i += MMW * 32) {
            const int m = i / n16, c = i - m * n16;
            *(int4 *)(sx + (size_t)m * kp + c * 16) = __ldcg((const int4 *)(gc + (size_t)m * K) + c);
        }
        for (int i = threadIdx.x; i < M * nb; i += MMW * 32) {
            const int m = i / nb, b = i - m * nb;
            sdh[m * dhs + b] = __half_as_ushort(__float2half_rn(__ldcg(gd + i)));  // the scales are f16 values: exact
            ss8[m * s8s + b] = __ldcg(gs + i);
        }
        named_bar(1, MMW * 32);
    }
    if (stamp) a.trace[blockIdx.x * 8 + 3] = global_ns();

    const int team = warp / MM_WPP, q = warp % MM_WPP;
    const int g = lane >> 2, tg = lane & 3;  // MMA fragment coordinates
    const int m = g;                          // this thread's activation row
    const int msrc = g < M ? g : 0;           // rows past M read row 0 (results dropped)
    float2 *myx = xch + (size_t)team * 2 * MM_MAXNR * 8 * 32;
    // A timed-out wait sets `ok` and skips the remaining pieces' work, but every warp of a team still
    // walks the same tiles and reaches the same named barriers.
    bool ok = true;
    for (int c0 = 0; c0 < L; c0 += MM_TEAMS) {
        const int n = c0 + MM_TEAMS < L ? MM_TEAMS : L - c0;
        if (team >= n) break;
        int mat, tile;
        gemv_piece(a, G, (int)blockIdx.x + (c0 + team) * (int)gridDim.x, 0, 0, &mat, &tile);
        const int row0 = tile * QTR + 2 * tg;  // this thread's weight rows row0, row0 + 1
        float e0[2] = {0.0f, 0.0f}, e1[2] = {0.0f, 0.0f};
        if (q == 0 && g < M) {
            mm_epi_load(a, mat, row0, m, e0[0], e1[0]);
            mm_epi_load(a, mat, row0 + 1, m, e0[1], e1[1]);
        }
        float acc[NR][8][2];
#pragma unroll
        for (int r = 0; r < NR; r++)
#pragma unroll
            for (int i = 0; i < 8; i++) acc[r][i][0] = acc[r][i][1] = 0.0f;
        const uint32_t tb = (uint32_t)(c0 * per_group);
        for (int s = 0; s < G.nseg; s++) {
            const int sb = (int)qw_seg_blocks(nb, s), rs = mm_row_stride(sb, CB), bbase = s * QSEG;
#pragma unroll
            for (int r = 0; r < NR; r++) {
                const uint32_t t = tb + (uint32_t)((s * n + team) * G.pieces + r);
                if (ok && !gemv_wait_piece(R, t)) ok = false;
                if (!ok) continue;
                const unsigned char *piece = R.data(t);
                const int ssh = mm_scale_stride(sb) / 2;  // halves between scale rows
                const uint16_t *scl = (const uint16_t *)(piece + QTR * rs);
                for (int u = 0; u < sb / 32; u++) {
                    const int j0 = 32 * u + 8 * q;  // this warp's 8 consecutive blocks of the segment
                    // the 8 blocks' scales of weight rows row0, row0 + 1 and the activation row's
                    uint4 w0s = *(const uint4 *)(scl + (2 * tg) * ssh + j0), w1s = *(const uint4 *)(scl + (2 * tg + 1) * ssh + j0);
                    const uint4 dxs = *(const uint4 *)(sdh + msrc * dhs + bbase + j0);
                    const uint16_t *sw0 = (const uint16_t *)&w0s, *sw1 = (const uint16_t *)&w1s, *sdx = (const uint16_t *)&dxs;
                    int s8v[8];
                    if (QT == 0) {
                        const int4 lo = *(const int4 *)(ss8 + msrc * s8s + bbase + j0), hi = *(const int4 *)(ss8 + msrc * s8s + bbase + j0 + 4);
                        s8v[0] = lo.x, s8v[1] = lo.y, s8v[2] = lo.z, s8v[3] = lo.w;
                        s8v[4] = hi.x, s8v[5] = hi.y, s8v[6] = hi.z, s8v[7] = hi.w;
                    }
                    // weight fragments: Q4_0 one ldmatrix.x4 per 4 blocks (16 nibble bytes a row);
                    // Q8_0 one per 2 blocks; row (lane % 8) of matrix (lane / 8)
                    uint32_t wb[8][2];
                    if (QT == 0) {
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            uint32_t w[4];
                            ldsm_x4(w, piece + (lane & 7) * rs + (j0 + 4 * h + (lane >> 3)) * 16);
#pragma unroll
                            for (int k = 0; k < 4; k++) {
                                wb[4 * h + k][0] = w[k] & 0x0f0f0f0fu;
                                wb[4 * h + k][1] = (w[k] >> 4) & 0x0f0f0f0fu;
                            }
                        }
                    } else {
#pragma unroll
                        for (int h = 0; h < 4; h++) {
                            uint32_t w[4];
                            ldsm_x4(w, piece + (lane & 7) * rs + (j0 + 2 * h + (lane >> 4)) * 32 + ((lane >> 3) & 1) * 16);
                            wb[2 * h][0] = w[0];
                            wb[2 * h][1] = w[1];
                            wb[2 * h + 1][0] = w[2];
                            wb[2 * h + 1][1] = w[3];
                        }
                    }
#pragma unroll
                    for (int h = 0; h < 4; h++) {  // activation fragments: one ldmatrix.x4 per 2 blocks
                        uint32_t x[4];
                        const int am = (lane & 7) < M ? (lane & 7) : 0;
                        ldsm_x4(x, sx + (size_t)am * kp + (bbase + j0 + 2 * h + (lane >> 4)) * 32 + ((lane >> 3) & 1) * 16);
#pragma unroll
                        for (int e = 0; e < 2; e++) {
                            const int i = 2 * h + e;  // chain 8q + i
                            int c0v, c1v;
                            mma_dot<QT>(c0v, c1v, x[2 * e], x[2 * e + 1], wb[i][0], wb[i][1]);
                            if (QT == 0) {
                                c0v -= s8v[i];
                                c1v -= s8v[i];
                            }
                            acc[r][i][0] = __fmaf_rn(mul_f16(sw0[i], sdx[i]), i2f_exact(c0v), acc[r][i][0]);
                            acc[r][i][1] = __fmaf_rn(mul_f16(sw1[i], sdx[i]), i2f_exact(c1v), acc[r][i][1]);
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&R.empty[R.slot(t)]);
            }
        }
        // chains across the team's warps, in the butterfly's pairs: level 16 (warps 2, 3 into 0, 1),
        // level 8 (warp 1 into 0), then 4, 2, 1 inside warp 0
        const int bar = 2 + team;
        if (q >= 2)
#pragma unroll
            for (int r = 0; r < NR; r++)
#pragma unroll
                for (int i = 0; i < 8; i++) myx[(((q - 2) * MM_MAXNR + r) * 8 + i) * 32 + lane] = make_float2(acc[r][i][0], acc[r][i][1]);
        named_bar(bar, MM_WPP * 32);
        if (q < 2)
#pragma unroll
            for (int r = 0; r < NR; r++)
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const float2 o = myx[((q * MM_MAXNR + r) * 8 + i) * 32 + lane];
                    acc[r][i][0] = __fadd_rn(acc[r][i][0], o.x);
                    acc[r][i][1] = __fadd_rn(acc[r][i][1], o.y);
                }
        named_bar(bar, MM_WPP * 32);
        if (q == 1)
#pragma unroll
            for (int r = 0; r < NR; r++)
#pragma unroll
                for (int i = 0; i < 8; i++) myx[((r * 8) + i) * 32 + lane] = make_float2(acc[r][i][0], acc[r][i][1]);
        named_bar(bar, MM_WPP * 32);
        if (q == 0) {
            float y[2][NR];
#pragma unroll
            for (int r = 0; r < NR; r++) {
                float c[2][8];
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const float2 o = myx[((r * 8) + i) * 32 + lane];
                    c[0][i] = __fadd_rn(acc[r][i][0], o.x);
                    c[1][i] = __fadd_rn(acc[r][i][1], o.y);
                }
#pragma unroll
                for (int nn = 0; nn < 2; nn++) {
#pragma unroll
                    for (int off = 4; off >= 1; off >>= 1)
#pragma unroll
                        for (int i = 0; i < off; i++) c[nn][i] = __fadd_rn(c[nn][i], c[nn][i + off]);
                    y[nn][r] = c[nn][0];
                }
            }
            if (g < M) {
                mm_epi<NR>(a, mat, row0, m, y[0], e0[0], e1[0]);
                mm_epi<NR>(a, mat, row0 + 1, m, y[1], e0[1], e1[1]);
            }
        }
        named_bar(bar, MM_WPP * 32);  // the exchange buffer is free for the next tile
    }
    if (!ok && a.err) atomicExch(a.err, 2);
    if (stamp) a.trace[blockIdx.x * 8 + 4] = global_ns();
}

bool g_mma_on = true, g_mma_read = false;

template <int QT, int NR>
void launch_mma(const FusedArgs &a, const GemvGeo &G, cudaStream_t s, bool pdl) {
    auto kern = gemv_mma_kernel<QT, NR>;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        attr = true;
    }
    constexpr int CB = QT == 0 ? 16 : 32;
    const int nb = (int)(a.K / 32), M = a.M;
    const int slot_bytes = mm_slot_bytes(QSEG < nb ? QSEG : nb, CB);
    size_t head = (size_t)2 * MM_MAXNS * 8 + (size_t)MM_TEAMS * 2 * MM_MAXNR * 8 * 32 * sizeof(float2);
    head += (size_t)M * (a.K + 16) + (size_t)M * mm_dh_stride(nb) * 2 + (size_t)M * mm_s8_stride(nb) * 4;
    head = (head + 127) / 128 * 128;
    int ns = ring_slots(224 * 1024, head, (size_t)slot_bytes, MM_MAXNS);
    if (ns < 2) throw std::runtime_error("gemv_mma: the staged rows leave no room for the weight ring");
    const size_t smem = head + (size_t)ns * slot_bytes;
    const int64_t cap = num_sms();
    const int64_t ctas = G.groups < cap ? (int64_t)G.groups : cap;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(ctas < 1 ? 1 : ctas));
    cfg.blockDim = dim3(MM_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a, G, ns, ring_magic((uint32_t)ns), slot_bytes);
    if (e != cudaSuccess) throw std::runtime_error(std::string("CUDA launch of gemv_mma failed: ") + cudaGetErrorString(e));
}

}  // namespace

bool gemv_mma_ok(const FusedArgs &a) {
    if (!g_mma_read) {
        if (const char *e = std::getenv("GCB_GEMV_MMA")) g_mma_on = std::atoi(e) != 0;
        g_mma_read = true;
    }
    const GemvGeo G = gemv_geo(a);
    return g_mma_on && a.M >= 2 && a.M <= 8 && a.pro == PRO_Q8 && a.xq && a.nshard == 1 && a.K % 1024 == 0 &&
           G.pieces <= MM_MAXNR && (a.qtype == T_Q4_0 || a.qtype == T_Q8_0);
}

void gemv_mma(const FusedArgs &a, cudaStream_t s, bool pdl) {
    const GemvGeo G = gemv_geo(a);
    const bool q4 = a.qtype == T_Q4_0;
    if (G.pieces == 1) {
        if (q4) launch_mma<0, 1>(a, G, s, pdl);
        else launch_mma<1, 1>(a, G, s, pdl);
    } else {
        if (q4) launch_mma<0, 2>(a, G, s, pdl);
        else launch_mma<1, 2>(a, G, s, pdl);
    }
}

}  // namespace k
}  // namespace gcb
