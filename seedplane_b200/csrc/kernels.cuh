// Kernel parameter blocks and host-side launchers of the decode kernels (kernels.cu).
#pragma once

#include "common.cuh"

namespace sp {

enum Prologue : int { PRO_PLAIN = 0, PRO_NORM = 1, PRO_EMBED_NORM = 2 };
enum Epilogue : int { EPI_QKV = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_LMHEAD = 3 };
enum WeightFmt : int { WF_F16 = 0, WF_I8 = 1 };

// One weight-streaming GEMV y = W . in(x) with a fused prologue and epilogue.
//   W is packed row-major [N][K] (fp16, or int8 + fp16 scales [N][K/32]); each CTA owns a
//   contiguous range of rows, streams it through a ring of shared-memory stages with 1-D bulk
//   copies (TMA engine), and reduces rows with warps (fp32 accumulation).
struct GemvParams {
    const uint8_t *w;
    const __half *ws;
    int N, K;
    int fmt;                 // WeightFmt
    int rows_per_chunk;      // R: rows per stage (multiple of the epilogue's row group)
    int split;               // segments per row (K/8 divisible by split)
    int stages;              // ring depth
    int stage_bytes;         // bytes per stage (128-aligned)
    int grid;                // CTAs (row ranges)
    // prologue
    const float *xin;
    const float *gain;
    const __half *embed;
    float *x_init;
    float eps;
    int vocab;
    // epilogue
    const float *bias;
    float *out;
    __half *kc, *vc;
    int cap;
    const float *rope;
    int max_pos;
    int nh, nkv, hd;
    // LM head
    float *part_val;
    int *part_idx;
    unsigned *counter;
    DevState *st;
};

struct AttnParams {
    const float *q;          // [NH*HD] fp32 (RoPE applied)
    const __half *kc, *vc;   // this layer's caches [NKV][cap][HD]
    float *out;              // [NH*HD] fp32
    float *part;             // [NH][max_split][HD+2] partial (m, l, acc)
    unsigned *counter;       // [NKV]
    int nh, nkv, hd, cap;
    int max_split, min_chunk;
    float scale;
    DevState *st;
};

struct LaunchCfg {
    cudaStream_t stream;
    bool pdl;                // launch with programmatic stream serialization
};

// Plan R / split / stages for a GEMV of N x K rows (row group `rg`); fills the geometry fields.
void plan_gemv(GemvParams &p, int rg, int num_sms, int ring_bytes);
size_t gemv_smem_bytes(const GemvParams &p);
// Set the dynamic shared-memory limit of the kernel instance (call before any stream capture).
cudaError_t prepare_gemv(int pro, int epi, const GemvParams &p);
cudaError_t launch_gemv(int pro, int epi, const GemvParams &p, const LaunchCfg &lc);
cudaError_t launch_attention(const AttnParams &p, const LaunchCfg &lc);

// Host-side launches of small utility kernels.
cudaError_t launch_set_state(DevState *st, const DevState &init, cudaStream_t s);
// dst row (r * dst_mul + dst_add) = src row src_row[r], for r < rows.
cudaError_t launch_gather_rows(uint8_t *dst, const uint8_t *src, const int *src_row, int rows, int row_bytes,
                               int dst_mul, int dst_add, cudaStream_t s);
cudaError_t launch_kv_commit(__half *k, __half *v, int layers, int nkv, int cap, int hd, const int *src_slots,
                             int n, int dst0, cudaStream_t s);

}  // namespace sp
