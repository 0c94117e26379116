// Per-op streamed quantized GEMV (decode, up to 8 activation rows), with its neighbouring nodes
// folded in (gc_fused.h: NORM / ACT prologue, SINGLE / ROPE_QKV / SWIGLU map, residual epilogue).
//
// Persistent CTAs, two per SM: warp 8 is the producer (one lane streams weight pieces with bulk
// copies into a ring of shared-memory slots, gc_gemv_dev.cuh), warps 0-7 are the consumers (one row
// of the current 8-row tile each). The producer reads nothing an earlier kernel writes and starts at
// once; the consumers execute griddepcontrol.wait (PDL) before reading the activation, and nothing is
// written before that wait. Every wait is bounded in time; a timeout sets the error word (2), the
// producer then waits (bounded) for its copies in flight, and the CTA exits.
#include <cstdlib>
#include <stdexcept>
#include <string>

#include "gc_gemv_dev.cuh"

namespace gcb {
namespace k {

namespace {

constexpr int NCW = 8;  // consumer warps
// One activation row: the 8 consumer warps are one team, one tile row each. Several rows: GEMV_RPW
// tile rows per warp (gc_gemv_dev.cuh consume_gemv), teams of 8 / GEMV_RPW warps, each team on its
// own row group, so each piece is released by the warps of one team.
#ifndef GEMV_RPW
#define GEMV_RPW 2
#endif
template <int M>
constexpr int teams_of() { return M == 1 ? 1 : GEMV_RPW; }
template <int M>
constexpr int threads_of() { return (NCW + 1) * 32; }
constexpr int MAXNS = 16;
constexpr int CG = 2;  // row groups per chunk with one activation row (gc_gemv_dev.cuh)

// One activation row: two CTAs per SM (96 registers). More rows: one CTA per SM, so the M x NR
// accumulators and the rows' operands stay in registers (at two per SM they spilled to local
// memory), with the whole shared memory for the staged rows and the ring.
template <int QT, int NR, int M>
__global__ void __launch_bounds__(threads_of<M>(), M == 1 ? 2 : 1) gemv_tma_kernel(FusedArgs a, GemvGeo G, int ns, uint32_t magic, int slot_bytes) {
    constexpr int TEAMS = teams_of<M>(), TW = NCW / TEAMS, NCT = NCW * 32;  // teams, warps per team, consumer threads
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t *full = (uint64_t *)smem;
    uint64_t *empty = full + MAXNS;
    uint64_t *hold = empty + MAXNS;          // the consumers' prologue is done (FusedArgs::hold_pieces)
    double *red = (double *)(hold + 2);      // [256]
    int8_t *sq = (int8_t *)(red + 256);
    float *sdf = (float *)(sq + (size_t)M * a.K);
    int *ss8 = (int *)(sdf + (size_t)M * G.nb);
    unsigned char *slots = (unsigned char *)(red + 256) + gemv_act_bytes(M, a.K);
    const Ring R{full, empty, slots, (uint32_t)ns, magic, slot_bytes};
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < ns; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], TW);
        }
        mbar_init(hold, 1);
        mbar_fence_init();
    }
    __syncthreads();
    pdl_trigger();

    if (warp == NCW) {  // producer
        if (lane != 0) return;
        if (a.trace) a.trace[blockIdx.x * 8 + 0] = global_ns();
        if (a.producer_waits) pdl_wait();
        uint32_t t = 0;
        if (!produce_gemv(a, G, R, t, blockIdx.x, gridDim.x, M == 1 ? gemv_chunk(1, 1, CG) : TEAMS,
                          a.hold_pieces > 0 ? hold : nullptr)) {
            if (a.err) atomicExch(a.err, 2);
            drain_ring(R, t);
        } else {
            if (a.trace) a.trace[blockIdx.x * 8 + 1] = global_ns();
            prefetch_next(a, blockIdx.x, gridDim.x);
        }
        return;
    }
    float4 wpre[GEMV_UB];
    gemv_norm_prefetch<NCT>(a, wpre);
    pdl_wait();
    const bool stamp = a.trace && threadIdx.x == 0;
    if (stamp) a.trace[blockIdx.x * 8 + 2] = global_ns();
    if (a.pro == PRO_Q8) gemv_stage_q8<NCT>(a, sq, 1, M);
    else gemv_prologue<M, NCT>(a, sq, sdf, ss8, red, 1, wpre);
    if (stamp) a.trace[blockIdx.x * 8 + 3] = global_ns();
    if (threadIdx.x == 0) mbar_arrive(hold);
    if (!consume_gemv<QT, NR, M, CG, TEAMS>(a, G, R, 0, blockIdx.x, gridDim.x, warp / TW, TEAMS, warp % TW, sq, sdf, ss8))
        if (a.err) atomicExch(a.err, 2);
    if (M == 1 && a.act_mode != ACT8_NONE) gemv_emit_act8<NCT>(a, G, red, 1);
    if (stamp) a.trace[blockIdx.x * 8 + 4] = global_ns();
}

// Activation rows -> Q8_0 blocks in the GEMV staging layout for M rows (gemv_act_bytes(M, K) bytes
// at dst: codes [M][K], f32 block scales [M][K / 32], 8 x code sums [M][K / 32]), with rms_norm x
// weight first for PRO_NORM: the consumers' prologue arithmetic, one CTA per row, done once for
// the launch that reads it (PRO_Q8) instead of in each of its CTAs.
__global__ void __launch_bounds__(256) act_rows_kernel(FusedArgs a, char *dst) {
    __shared__ double red[256];
    pdl_trigger();
    pdl_wait();  // the rows were written by the kernel before
    const int m = blockIdx.x, nb = (int)(a.K / 32);
    FusedArgs r = a;
    r.x = a.x + (int64_t)m * a.ldx;
    r.M = 1;
    int8_t *codes = (int8_t *)dst;
    float *d = (float *)(dst + (size_t)a.M * a.K);
    int *s8 = (int *)(d + (size_t)a.M * nb);
    gemv_prologue<1, 256>(r, codes + (size_t)m * a.K, d + (size_t)m * nb, s8 + (size_t)m * nb, red, 1);
}

int g_num_sms = 0;
size_t g_smem_budget = 0;
int g_ctas_per_sm = 2;  // GCB_GEMV_CTAS_PER_SM: 1 leaves room for the next launch's CTAs (PDL)

template <int QT, int NR, int M>
void launch_t(const FusedArgs &a, const GemvGeo &G, cudaStream_t s, bool pdl) {
    auto kern = gemv_tma_kernel<QT, NR, M>;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        attr = true;
    }
    const int slot_bytes = (int)qw_piece_bytes(G.nb, G.cb, 0);
    const size_t head = (size_t)(2 * MAXNS + 2) * 8 + 256 * 8 + gemv_act_bytes(M, a.K);
    const size_t budget = g_smem_budget ? g_smem_budget : (M == 1 && g_ctas_per_sm == 2 ? 113 * 1024 : 224 * 1024);
    int ns = ring_slots(budget, head, (size_t)slot_bytes, MAXNS);
    if (ns < 2 * G.pieces) ns = 2 * G.pieces;  // room for one group's pieces in flight and one consumed
    const size_t smem = head + (size_t)ns * (size_t)slot_bytes;
    const int per_sm = M == 1 && smem <= 113 * 1024 ? g_ctas_per_sm : 1;
    const int64_t cap = (int64_t)g_num_sms * per_sm;
    int64_t ctas = G.groups < cap ? (int64_t)G.groups : cap;
    if (a.max_ctas > 0 && ctas > a.max_ctas) ctas = a.max_ctas;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(ctas < 1 ? 1 : ctas));
    cfg.blockDim = dim3(threads_of<M>());
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a, G, ns, ring_magic((uint32_t)ns), slot_bytes);
    if (e != cudaSuccess) throw std::runtime_error(std::string("CUDA launch of gemv_tma failed: ") + cudaGetErrorString(e));
}

template <int QT, int NR>
void launch_m(const FusedArgs &a, const GemvGeo &G, cudaStream_t s, bool pdl) {
    switch (a.M) {
        case 1: launch_t<QT, NR, 1>(a, G, s, pdl); break;
        case 2: launch_t<QT, NR, 2>(a, G, s, pdl); break;
        case 3: launch_t<QT, NR, 3>(a, G, s, pdl); break;
        case 4: launch_t<QT, NR, 4>(a, G, s, pdl); break;
        case 5: launch_t<QT, NR, 5>(a, G, s, pdl); break;
        case 6: launch_t<QT, NR, 6>(a, G, s, pdl); break;
        case 7: launch_t<QT, NR, 7>(a, G, s, pdl); break;
        case 8: launch_t<QT, NR, 8>(a, G, s, pdl); break;
        default: throw std::runtime_error("gemv_tma: 1 to 8 activation rows");
    }
}

}  // namespace

int num_sms() {
    if (!g_num_sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (const char *b = std::getenv("GCB_GEMV_SMEM_KB")) g_smem_budget = (size_t)std::atoi(b) * 1024;
        if (const char *c = std::getenv("GCB_GEMV_CTAS_PER_SM")) g_ctas_per_sm = std::atoi(c) == 1 ? 1 : 2;
    }
    return g_num_sms;
}

bool fused_gemv_supported(int64_t K, int64_t M, int map) {
    (void)map;
    if (K % 32 || M < 1 || M > GEMV_MAXM) return false;
    return gemv_act_bytes((int)M, K) <= 64 * 1024;
}

void act_rows(const FusedArgs &a, char *dst, cudaStream_t s) {
    if (a.pro != PRO_ACT && a.pro != PRO_NORM) throw std::runtime_error("act_rows: f32 rows in (ACT or NORM prologue)");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)a.M);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, act_rows_kernel, a, dst);
    if (e != cudaSuccess) throw std::runtime_error(std::string("CUDA launch of act_rows failed: ") + cudaGetErrorString(e));
}

bool fused_gemv_args_ok(const FusedArgs &a) { return a.map != MAP_ROPE_QKV || (a.D / 2) % QTR == 0; }

void fused_gemv(const FusedArgs &a, cudaStream_t s, bool pdl) {
    num_sms();
    if (!fused_gemv_args_ok(a)) throw std::runtime_error("gemv_tma: head size must be a multiple of 16");
    if (gemv_mma_ok(a)) {
        gemv_mma(a, s, pdl);
        return;
    }
    const GemvGeo G = gemv_geo(a);
    const bool q4 = a.qtype == T_Q4_0;
    if (G.pieces == 1) {
        if (q4) launch_m<0, 1>(a, G, s, pdl);
        else launch_m<1, 1>(a, G, s, pdl);
    } else {
        if (q4) launch_m<0, 2>(a, G, s, pdl);
        else launch_m<1, 2>(a, G, s, pdl);
    }
}

}  // namespace k
}  // namespace gcb
