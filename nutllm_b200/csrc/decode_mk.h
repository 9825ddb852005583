#pragma once
/* The persistent token-loop kernel (one launch per generation). */
#include <cstdint>
#include <cuda_runtime.h>

#include "kernels_tc.h"

namespace nut {

/* Weights of one layer in fragment tiles. */
struct MkLayer {
    TileMatrix qkv;  /* [dim + 2 kv_dim][dim]: query, key, value rows,
                        row-major tiles */
    TileMatrix wo;   /* [dim][dim], pair-column tiles (split by K pairs) */
    TileMatrix gu;   /* [2 ffn][dim]: gate and up rows interleaved in groups
                        of 8 (a 16-row tile = gate 8t..8t+7, up 8t..8t+7),
                        row-major tiles */
    TileMatrix down; /* [dim][ffn], block-column tiles (split by K blocks) */
};

/* Accumulator slots of the split-K reductions (a ring; see decode_mk.cu). */
constexpr int kAccSlots = 8;
/* Most FFN blocks (32 hidden units) whose Wdown columns one CTA may own. */
constexpr int kMaxFfnBlocks = 4;
/* Row-tile pairs of one Wdown work unit (a column block is split into units
 * of this many pairs). */
constexpr int kDownUnitPairs = 32;

/* FFN work units of one 32-unit block: its 4 gate/up row tiles, then its
 * Wdown column block in units of kDownUnitPairs row-tile pairs. */
inline int ffn_units_per_block(int rt_down_pairs) {
    return 4 + (rt_down_pairs + kDownUnitPairs - 1) / kDownUnitPairs;
}

/* Device-side view of a layer (pointers only). */
struct MkLayerPtrs {
    const uint8_t *qkv, *wo, *gu, *down;
    const uint16_t *qkv_s, *wo_s, *gu_s, *down_s;
};

/* Cross-CTA tagged vector element: value bits in .x, tag in .y, written and
 * read as one 64-bit access. */
using Tagged = uint2;

/* Words per phase record of the optional trace. */
constexpr int kTraceWords = 16;

struct MkParams {
    int layers, dim, kvd, heads, kv_heads, hd, ffn, vocab, max_seq;
    int nb_dim, nb_ffn;                 /* padded blocks of K = dim / ffn */
    int rt_qkv, rt_wo, rt_gu, rt_down;  /* row tiles per matrix */
    const MkLayerPtrs *layer;           /* [layers] */
    const float *attn_norm, *ffn_norm;  /* [layers][dim] */
    const float *final_norm;            /* [dim] */
    const float *lm_head;               /* [vocab][dim] (embeddings if tied) */
    const float *emb;                   /* [vocab][dim] */
    const float *rope_cos, *rope_sin;   /* [max_seq][hd / 2] */
    float *kcache, *vcache;             /* [layers][kv_heads][max_seq][hd] */
    Tagged *qkv;                        /* tagged q | k | v of the current token */
    Tagged *act;                        /* [ffn] tagged SwiGLU outputs that cross
                                           CTAs */
    float *hacc;                        /* [kAccSlots][dim] residual stream
                                           accumulators (fp32, red.add) */
    float *hidden_out;                  /* [dim] last hidden vector */
    unsigned int *cnt;                  /* [kAccSlots] contributions counted */
    int wo_pairs, cpp;                  /* K pairs of Wo; CTAs per pair */
    int count_aw;                       /* CTAs of the attention + Wo step */
    int nbf, count_gd;                  /* FFN blocks; CTAs of the FFN step */
    int rt_down_pairs;                  /* row-tile pairs per Wdown block */
    int gd_unit, gd_total;              /* FFN work units per block, in all */
    const int *prompt;                  /* [n_prompt] */
    int n_prompt, n_tokens, start_pos;
    int logits_from, logits_to;         /* lm_head after tokens in [from, to] */
    unsigned long long *keys;           /* [n_tokens] argmax keys */
    unsigned int *done;                 /* [n_tokens] CTAs done with lm_head */
    float *logits;                      /* [to - from + 1][vocab] or null */
    int *error;
    unsigned long long *stamps;         /* [3] start, prefill done, end (ns) */
    unsigned long long *trace;          /* optional [ctas][trace_stride][kTraceWords] */
    int trace_stride;
    uint64_t limit_ns;
    int att_chunk;                      /* positions per attention chunk */
    int union_floats;                   /* floats in the digits/attention union */
    Tagged *xchg;                       /* [count_aw][hd + 2] tagged partial
                                           attention states of split histories
                                           (the LONG kernel) */
};

/* Launches the kernel cooperatively on `stream`.  Returns the launch
 * status; device-side failures land in *p.error. */
cudaError_t launch_decode_mk(const MkParams &p, int type, int sms, cudaStream_t stream);

/* Whether a model shape can run the persistent kernel on this device. */
bool mk_supported(int dim, int ffn, int kvd, int head_dim, int heads, int type,
                  int max_smem, int sms);

} // namespace nut
