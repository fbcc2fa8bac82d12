// Internal declarations shared by the .cu translation units of libgtmoe.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>

#include "gtmoe.h"

namespace gtm {

int set_error(int status, const char* fmt, ...);
int set_cuda_error(const char* what, cudaError_t e);
void clear_error();

size_t decode_workspace_bytes();
size_t decode_sticky_offset();
constexpr int kDecodeMinCtas = 120;   // per-CTA work lists of the fused decode fit its slot arrays
int launch_decode(const GtmDims& dims, const GtmLayer* layers, int num_layers, const GtmDecodeIO& io,
                  void* ws, size_t ws_bytes, cudaStream_t stream, int num_ctas);

size_t lm_head_workspace_bytes(uint32_t rows);
int launch_lm_head(uint32_t rows, const void* w, const uint16_t* s, const uint16_t* b, const float* x, uint32_t* token,
                   float* logit, void* ws, cudaStream_t st, int num_sms);
int lm_head_candidates(void* ws, cudaStream_t st, int* n);

size_t tokens_workspace_bytes(uint32_t max_tokens);
int launch_tokens(const GtmDims& dims, const GtmLayer& layer, const GtmTokensIO& io, void* ws, size_t ws_bytes,
                  cudaStream_t stream, int num_sms);
int tokens_check(void* ws, cudaStream_t stream);
int set_phase_events(void* const* events, int n);
size_t ep_workspace_bytes(uint32_t max_tokens, uint32_t max_recv);
int launch_ep_dispatch(const GtmDims& dims, const GtmLayer& L, const GtmTokensIO& io, const GtmEpConfig& ep,
                       float* send_rows, GtmEpMeta* send_meta, int32_t* send_counts, void* ws, cudaStream_t st);
int launch_ep_shared(const GtmLayer& L, const GtmTokensIO& io, const GtmEpConfig& ep, void* ws, cudaStream_t st,
                     int num_sms, bool peer);
int launch_ep_experts(const GtmLayer& L, const GtmEpConfig& ep, const float* recv_rows, const GtmEpMeta* recv_meta,
                      uint32_t n_recv, float* ret_rows, void* ws, cudaStream_t st, int num_sms);
int launch_ep_combine(const GtmDims& dims, const GtmLayer& L, const GtmTokensIO& io, const GtmEpConfig& ep,
                      const float* ret_rows, void* ws, cudaStream_t st);
size_t ep_peer_workspace_bytes(uint32_t world, uint32_t max_tokens);
int launch_ep_peer_dispatch(const GtmDims& dims, const GtmLayer& L, const GtmTokensIO& io, const GtmEpConfig& ep,
                            void* const* peer_ws, cudaStream_t st);
int launch_ep_peer_experts(const GtmLayer& L, const GtmEpConfig& ep, void* const* peer_ws, cudaStream_t st,
                           int num_sms);
int launch_ep_peer_combine(const GtmDims& dims, const GtmLayer& L, const GtmTokensIO& io, const GtmEpConfig& ep,
                           void* ws, cudaStream_t st);

// generic kernels (gtm_kernels.cu); arguments already validated
void k_gemv_exact(int bits, uint32_t rows, uint32_t in_dim, const void* w, const uint16_t* s, const uint16_t* b,
                  const float* x, float* out, uint32_t row_begin, uint32_t row_end, cudaStream_t st,
                  uint32_t nvec = 1);
// int4 rows of n >= 2 vectors (x 16-byte aligned), the same results as k_gemv_exact per vector;
// false (nothing launched) when in_dim is outside its shapes
bool k_gemv_exact_rows4(uint32_t rows, uint32_t in_dim, uint32_t n, const void* w, const uint16_t* s, const uint16_t* b,
                        const float* x, float* out, cudaStream_t st);
void k_router_topk(uint32_t n, uint32_t k, const float* logits, const uint16_t* pes, uint32_t* idx, float* w,
                   cudaStream_t st);
void k_geglu(uint32_t n, const float* g, const float* u, float* out, cudaStream_t st);
void k_scale_accum(uint32_t n, const float* in, const float* w, uint32_t wi, int acc, float* out, cudaStream_t st);
void k_mul_bf16(uint32_t n, const float* in, const uint16_t* w, float scale, float* out, cudaStream_t st);
void k_rmsnorm(uint32_t n, const float* x, const uint16_t* w, float eps, float* out, cudaStream_t st,
               uint32_t rows = 1);
void k_post_attn(uint32_t d, const float* attn, const float* hidden, const uint16_t* wpost, const uint16_t* wpre,
                 const uint16_t* wpre2, float eps, float* hout, float* dense, float* routed, float* router,
                 cudaStream_t st, uint32_t rows = 1);
void k_layer_tail(uint32_t d, const float* h2, const float* h1, const float* hidden, const uint16_t* wpf2,
                  const uint16_t* wpf, float eps, float ls, float* hout, cudaStream_t st);

constexpr uint32_t kMaxNormDim = 16384;   // vectors normalised in one CTA's shared memory
constexpr uint32_t kMaxBatchRows = 512;    // vectors of one *_rows call (per-row arguments travel by value)

}  // namespace gtm
