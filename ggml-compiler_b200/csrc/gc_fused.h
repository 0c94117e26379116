// Arguments of the fused decode GEMV kernel (kernels/gc_fused.cu).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "gc_types.h"

namespace gcb {

// The activation prologue: quantize the f32 row(s) (PRO_ACT), rms_norm x weight first (PRO_NORM),
// or take Q8_0 blocks a kernel before wrote in the staging layout (PRO_Q8).
enum { PRO_ACT = 0, PRO_NORM = 1, PRO_Q8 = 2 };
// What a launch emits for the GEMV after it (one row): nothing, the rms_norm-ed output row's Q8_0
// blocks (written by the launch's last CTA), or the output's own Q8_0 blocks (each written by the
// CTA that stores the block's last 8-row tile).
enum { ACT8_NONE = 0, ACT8_NORM = 1, ACT8_BLOCKS = 2 };
enum { MAP_SINGLE = 0, MAP_ROPE_QKV = 1, MAP_SWIGLU = 2 };

struct FusedArgs {
    int qtype = T_Q4_0;  // of every weight
    int pro = PRO_ACT;
    int map = MAP_SINGLE;
    // activation rows: x[m * ldx + k], m < M, k < K
    const float *x = nullptr;
    int64_t ldx = 0;
    int M = 1;
    int64_t K = 0;
    const float *norm_w = nullptr;  // PRO_NORM
    float eps = 0.0f;
    // PRO_Q8: the M rows in the consumers' staging layout (gemv_act_bytes(M, K) bytes: int8 codes
    // [M][K], f32 block scales [M][K / 32], int 8 x code sums [M][K / 32]), written by the kernel before
    const char *xq = nullptr;
    // ACT8_NORM / ACT8_BLOCKS: where this launch writes the next GEMV's row in that layout, the
    // next GEMV's norm weight and eps (ACT8_NORM), and zeroed counters the launch leaves zero (one
    // for ACT8_NORM, one per 32-row block for ACT8_BLOCKS)
    int act_mode = ACT8_NONE;
    char *act_out = nullptr;
    const float *act_norm_w = nullptr;
    float act_eps = 0.0f;
    int *act_cnt = nullptr;
    // weights: repacked codes + fp16 scales, rows of K
    const char *wc[3] = {nullptr, nullptr, nullptr};
    const uint16_t *ws[3] = {nullptr, nullptr, nullptr};
    int64_t wrows[3] = {0, 0, 0};
    // MAP_SINGLE / MAP_SWIGLU output, optional residual (MAP_SINGLE)
    float *out = nullptr;
    int64_t ldo = 0;
    const float *res = nullptr;
    int64_t ldr = 0;
    // MAP_ROPE_QKV
    int64_t D = 0, H = 0, Hkv = 0;
    float *q_out = nullptr;
    int64_t ldq = 0;
    char *kcache = nullptr, *vcache = nullptr;
    int64_t cache_nb1 = 0, cache_nb2 = 0, cache_rows = 0;
    // bytes between the caches of consecutive activation rows: 0 when every row is a token of one
    // sequence; a sequence slot's size when row m is sequence m of a batched decode step
    int64_t cache_nb3 = 0;
    const int32_t *pos = nullptr;
    const float *table = nullptr;
    int64_t npos = 0;
    float theta_scale = 1.0f;
    int *err = nullptr;
    // Tensor-parallel shard: this launch computes shard `shard` of `nshard` of the rows (a run of
    // 8-row tiles; for MAP_ROPE_QKV the query and K/V heads H / nshard * shard.., Hkv / nshard * shard..).
    int shard = 0, nshard = 1;
    // Weights that a later kernel of the step streams: the leading bytes of up to three matrices,
    // fetched into L2 by this launch's producers once they have issued their own pieces (each
    // range split evenly over the CTAs), so HBM keeps streaming through this launch's tail, the
    // launch gap and the next launch's prologue. Addresses 16-byte aligned, sizes multiples of 256.
    const char *pf[3] = {nullptr, nullptr, nullptr};
    int64_t pf_bytes[3] = {0, 0, 0};
    int stream_evict_first = 0;  // stream this launch's weights under an L2 evict-first policy
    // GGML_COMPILER_B200_TRACE: %globaltimer stamps per CTA, [CTA][8] (k::kTraceSlots): producer
    // start, producer done issuing, consumers past the dependent-launch wait, prologue done,
    // consumers done (epilogue included). Null: no stamps.
    uint64_t *trace = nullptr;
    // The producer issues this many pieces, then waits (bounded) until the consumers' prologue is
    // done before issuing the rest, so that the prologue's loads do not queue behind the ring's
    // fill. 0: no wait.
    int hold_pieces = 0;
    // The producer waits for the previous kernel to complete (griddepcontrol.wait) before it
    // streams, instead of streaming during that kernel's latency-bound tail.
    int producer_waits = 0;
    // At most this many CTAs (0: two per SM, or one when the shared memory needs it). One per SM
    // leaves each SM room for a CTA of the attention launched after this GEMV, which can then
    // start its K/V copies while this GEMV runs.
    int max_ctas = 0;
};

namespace k {
int num_sms();  // of the current device
bool fused_gemv_supported(int64_t K, int64_t M, int map);
// Shape preconditions of one set of arguments (the rope map needs head sizes that are multiples of 16).
bool fused_gemv_args_ok(const FusedArgs &a);
void fused_gemv(const FusedArgs &a, cudaStream_t s, bool pdl);
// 2-8 staged activation rows (PRO_Q8), K a multiple of 1024, one shard: the block dots on the tensor
// cores (kernels/gc_gemv_mma.cu), the same results; fused_gemv takes this path when it applies
// (GCB_GEMV_MMA=0: never).
bool gemv_mma_ok(const FusedArgs &a);
void gemv_mma(const FusedArgs &a, cudaStream_t s, bool pdl);
// a's M activation rows (x, ldx, K; normed for PRO_NORM) into the PRO_Q8 staging layout for M
// rows at dst (gemv_act_bytes(M, K) bytes), one CTA per row: the launch that reads them then only
// copies them into shared memory.
void act_rows(const FusedArgs &a, char *dst, cudaStream_t s);
}  // namespace k

}  // namespace gcb
