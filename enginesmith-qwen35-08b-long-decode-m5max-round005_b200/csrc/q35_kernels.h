// Host-side launchers of the q35 decode kernels (implemented in q35_kernels.cu).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

#include "q35_types.h"

namespace q35 {

cudaError_t kernels_init();
// Byte offset of the bounded-wait error word in a q35_op_qgemm_q4 workspace.
size_t qgemm_err_offset();
// Scratch base of the allocation-free attention op on device `dev` (NULL
// before that op's first call there).
unsigned char* noalloc_scratch(int dev);
// Largest rows-per-CTA whose k_qmv shared-memory layout fits one CTA per SM.
int qmv_max_rows(int K);
size_t qmv_smem_bytes(const QmvArgs& a);
size_t attn_smem_bytes();
size_t head_smem_bytes();

cudaError_t launch_qmv(const QmvArgs& a, cudaStream_t st, bool pdl);
cudaError_t launch_recur(const RecurArgs& a, cudaStream_t st, bool pdl);
cudaError_t launch_attn(const AttnArgs& a, cudaStream_t st, bool pdl);
cudaError_t launch_head(const HeadArgs& a, cudaStream_t st, bool pdl);
cudaError_t launch_head_batch(const HeadBatchArgs& a, cudaStream_t st, bool pdl);
cudaError_t launch_greedy(const HeadArgs& a, cudaStream_t st);
cudaError_t launch_gdn_conv(const uint16_t* raw, uint16_t* hist, const uint16_t* convw,
                            uint16_t* conv_out, cudaStream_t st);
cudaError_t launch_ctl_position(Ctl* ctl, uint32_t pos, cudaStream_t st);
cudaError_t launch_greedy_sessions(const HeadOut* outs, int n, cudaStream_t st, bool pdl);
cudaError_t launch_attn_sessions(const AttnArgs& a, int n, cudaStream_t st, bool pdl);
cudaError_t launch_wait_probe(uint32_t polls, uint32_t* err, cudaStream_t st);

// Per-token steps of the tensor-core batched route (q35_tokens.cu)
cudaError_t launch_tok_rms(const TokArgs& a, cudaStream_t st, bool pdl);
cudaError_t launch_tok_conv(const TokArgs& a, cudaStream_t st, bool pdl);
cudaError_t launch_tok_normgate(const TokArgs& a, cudaStream_t st, bool pdl);
cudaError_t launch_tok_swiglu(const TokArgs& a, cudaStream_t st, bool pdl);

// Q4 GEMM on the tensor cores (q35_gemm.cu)
cudaError_t qgemm_init();
// TMA descriptors: 2-D (inner extent d0 contiguous, d1 rows `pitch` bytes
// apart) and 3-D (pitches p1, p2 of dims 1 and 2), boxes b0 x b1 (x b2)
bool tmap_2d(CUtensorMap* m, CUtensorMapDataType ty, const void* base, uint64_t d0, uint64_t d1,
             uint64_t pitch, uint32_t b0, uint32_t b1, CUtensorMapSwizzle sw);
bool tmap_3d(CUtensorMap* m, CUtensorMapDataType ty, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
             uint64_t p1, uint64_t p2, uint32_t b0, uint32_t b1, uint32_t b2, CUtensorMapSwizzle sw);
size_t qgemm_workspace_bytes(int N, int K, int T);
size_t qgemm_workspace_bytes(const QGemmArgs& a);
cudaError_t launch_qgemm(QGemmArgs a, void* ws, size_t ws_bytes, bool zero_counters, cudaStream_t st,
                         bool pdl);

// prompt chunks on the tensor cores (q35_prompt.cu)
cudaError_t prompt_kernels_init();
size_t prompt_attn_items_max(int tmax, uint32_t capacity);
void prompt_attn_plan(PromptArgs& a);  // query blocks and key splits of the chunk
cudaError_t launch_prompt_rope(uint32_t p0, int T, float* rope, cudaStream_t st, bool pdl);
cudaError_t launch_prompt_conv(const PromptArgs& a, cudaStream_t st, bool pdl);
cudaError_t launch_prompt_gdn_prep(const PromptArgs& a, cudaStream_t st, bool pdl);
cudaError_t launch_prompt_recur(const PromptArgs& a, cudaStream_t st, bool pdl);
cudaError_t launch_prompt_attn_prep(const PromptArgs& a, cudaStream_t st, bool pdl);
cudaError_t launch_prompt_attn(PromptArgs a, cudaStream_t st, bool pdl);

// prompt chunks (q35_prefill.cu)
cudaError_t chunk_kernels_init();
int chunk_sub_tokens(const QmvArgs& a);  // tokens per shared-memory sub-chunk
cudaError_t launch_qmv_chunk(const QmvArgs& a, cudaStream_t st, bool pdl);
cudaError_t launch_recur_chunk(const RecurArgs& a, cudaStream_t st, bool pdl);
cudaError_t launch_recur_sessions(const RecurArgs& a, int n, cudaStream_t st, bool pdl);
cudaError_t launch_embedding(const uint32_t* w, const uint16_t* s, const uint16_t* b,
                             uint32_t token, int K, uint16_t* out, cudaStream_t st);
cudaError_t launch_rms1024(const uint16_t* x, const uint16_t* gain, uint16_t* out,
                           cudaStream_t st);

}  // namespace q35
