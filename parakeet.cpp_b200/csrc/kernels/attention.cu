// Dispatcher of the relative-position attention (the tcgen05 kernel in
// attention_tc.cu). Reference: RelPosAttention::build_graph_batched
// (src/relpos_attention.cpp:162-306).
#include "kernels.h"

namespace pkc {

int attn_query_tile() { return attn_tc_query_tile(); }

cudaError_t attention_launch(const AttnArgs& a, bool bf16, cudaStream_t st) {
  return attention_tc_launch(a, bf16, st);
}

}  // namespace pkc
