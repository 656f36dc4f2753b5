// va_tc.cuh -- host interface of the tensor-core candidate filter (va_tc.cu).
#pragma once
#include <stdint.h>

struct va_context;

// Work decomposition of one filter launch: (query tile of 128) x (row split) items, statically
// strided over a persistent grid of at most one CTA per SM.
// Levels of the shared per-query bound (see the filter kernel): level l has `slots[l]` slots
// starting at slot `off[l]`, fed with the key at list rank `rank[l]`; slots[l] * rank[l] is at
// least the final pool. n = 0 means one level of one slot at rank kp.
struct BoundLevels {
    int n;
    int slots[4];
    int rank[4];
    int off[4];
};

struct TcPlan {
    int n_qtiles;
    int n_tiles;
    int splits;
    int kp;       // per-query candidate list length
    int grid;
    bool pair;    // cta_group::2 pair kernel (query tiles of 256), else single-CTA (128)
    int64_t nq_pad;
    int chunk_tiles;     // lockstep pacing: row tiles per chunk
    int lag;             // chunks a CTA may run ahead of the slowest
    int cpr;             // chunk slots per round
    int64_t sync_words;  // size of the pacing counter array
    int bound_slots;     // shared-bound slots per query, all levels (the gthr array's height)
    BoundLevels levels;  // va_tc_plan: one slot at rank kp; va_tc_plan_pool: up to four levels
};

struct TcFilterArgs {
    const void* q_op;     // queries, [nq_pad x dpad] bf16 or fp32, zero padded
    const void* x_op;     // rows, [n_rows x dpad] bf16 or fp32, zero padded
    int elem_bytes;       // 1 = int8 (kind::i8, exact), 2 = bf16 (kind::f16), 4 = fp32 as tf32 (kind::tf32)
    int64_t dpad;         // padded row length in elements (multiple of 64)
    int64_t n_rows;
    const float* row_bias;  // per row: |x|^2 (L2) or 0 (IP, cosine); +inf for the rows past n_rows
                            // up to a multiple of 256 (those never pass the filter)
    float alpha;            // key = alpha * dot + row_bias (float operands)
    const int* row_qn;      // int8 operands: per query |code|^2 (or |code| of 0/1 codes); the key is
                            // then the exact integer row_bias - 2 * dot + row_qn (row_bias holds ints)
    float* part_keys;       // [splits][nq_pad][kp]
    uint32_t* part_ids;     // [splits][nq_pad][kp]
    uint32_t* gthr;         // [total slots][nq_pad] shared per-query bound slots (orderable keys),
                            // set to 0xFF bytes by va_tc_filter
    uint32_t* sync_cnt;     // [sync_words] pacing counters, zeroed by va_tc_filter
    int64_t sync_words;
    unsigned limit_ms;    // bound of every device-side wait
    BoundLevels levels;   // bound levels (levels.n = 0: one slot at rank kp); every level's
                          // slots * rank must be at least the final pool (kp when the pool is the list)
};

// row_bytes: bytes of one operand row (dpad x element size), which sets the time of a tile.
int va_tc_plan(va_context* ctx, int64_t nq, int64_t n_rows, int kp, TcPlan* plan, int64_t row_bytes = 1536);
int va_tc_plan_pool(va_context* ctx, int64_t nq, int64_t n_rows, int pool, TcPlan* plan, int64_t row_bytes = 1536);
int va_tc_filter(va_context* ctx, const TcFilterArgs& a, const TcPlan& p);
int va_tc_stages(int kp, bool pair);
bool va_tc_use_pair();
// List mode (IVF list scan): query tile i against the rows [list_off[L], list_off[L+1]) of list
// L = tile_list[i] (device arrays); this launch runs tiles [tile0, tile0 + tiles) of n_qtiles;
// lists out as [n_qtiles * 128][kp]; a.sync_cnt unused. Row r of the query tiles is (query,
// probe) pair row_pair[r] (-1: padding) of query row_pair[r] / pair_div; the shared bound is per
// query, reset before the launch when reset_bounds (else kept from the previous launch).
int va_tc_filter_lists(va_context* ctx, const TcFilterArgs& a, int n_qtiles, int tile0, int tiles,
                       const int* tile_list, const int64_t* list_off, const int* row_pair, int pair_div, int kp,
                       bool reset_bounds);
