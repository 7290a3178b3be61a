// prefill_tc.cu -- varlen causal prefill on tcgen05 tensor cores (placeholder
// until the kernel lands: reports the shape as unsupported so the CUDA-core
// kernel runs).
#include "zl_internal.h"

namespace zl {

zl_status launch_prefill_tc(zl_ctx* ctx, const void* q, const void* k, const void* v,
                            const int32_t* cu_seqlens, int num_seqs, int max_seq_len, void* out,
                            int H, int Hkv, int d, float scale, int causal, zl_gqa_map map,
                            cudaStream_t st) {
  (void)ctx; (void)q; (void)k; (void)v; (void)cu_seqlens; (void)num_seqs; (void)max_seq_len;
  (void)out; (void)H; (void)Hkv; (void)d; (void)scale; (void)causal; (void)map; (void)st;
  return ZL_ERR_UNSUPPORTED;
}

}  // namespace zl
