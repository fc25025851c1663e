// q3cu_internal.h -- launchers shared between the kernel files and the C ABI.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "q3cu.h"
#include "q3cu_device.cuh"

namespace q3 {

// Context internals for the other translation units of the library.
q3cu_status set_error(q3cu_status s, const char *msg);   // records msg for q3cu_last_error_string
bool ctx_alive(const q3cu_ctx *ctx);
q3cu_status ctx_use_device(q3cu_ctx *ctx);                // makes the context's device current
int ctx_sms(const q3cu_ctx *ctx);
uint32_t *ctx_status_word(const q3cu_ctx *ctx);               // the device status word (Q3CU_DEV_* bits)

// Raises a kernel's dynamic shared-memory limit once per (device, slot):
// `slot` (< 32) names the kernel instantiation.
cudaError_t ensure_smem_attr(const void *kernel, size_t bytes, int slot);

// Launches `kernel` as a programmatic dependent of the stream's previous
// kernel: its CTAs may start before that kernel has completed, so the kernel
// calls griddep_wait() before it reads or writes any global memory that an
// earlier launch writes or reads (every thread that does, on every path), and
// griddep_launch_dependents() where its own successor may start.  When the
// previous work is not a kernel the launch behaves as an ordinary one.
template <typename... KArgs, typename... Args>
cudaError_t launch_dependent(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                             Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// The failure-path self-test: one CTA whose bounded wait on a barrier that
// nothing completes gives up and sets Q3CU_DEV_TIMEOUT in `status`.
cudaError_t launch_selftest_wait(uint32_t *status, cudaStream_t stream);

// Every launcher enqueues on `stream`, allocates nothing and returns the
// launch error.  `sms` is the device's multiprocessor count (grid sizing).
cudaError_t launch_quantize_q8(const void *x, q3cu_dtype dt, int64_t elems, int8_t *q, float *s,
                               cudaStream_t stream, int sms);
cudaError_t launch_dequantize_q8(const int8_t *q, const float *s, int64_t n, float *x, cudaStream_t stream,
                                 int sms);
cudaError_t launch_embed_gather(const int8_t *tq, const float *ts, int vocab, int dim, const int32_t *ids,
                                int64_t n, float *out, int8_t *oq, float *os, uint32_t *status,
                                cudaStream_t stream, int sms);

cudaError_t launch_rmsnorm(const void *x, q3cu_dtype dt, const float *w, int64_t rows, int dim, float eps,
                           void *out, int8_t *q, float *s, uint32_t *status, cudaStream_t stream, int sms);

cudaError_t launch_rmsnorm_padded(const float *x, const float *w, int size, int padded, float *out, uint32_t *status,
                                  cudaStream_t stream, int sms);

struct InvFreq { float v[64]; };
cudaError_t launch_qk_norm_rope(void *q, void *k, q3cu_dtype dt, const int32_t *pos, int64_t rows, int n_heads,
                                int n_kv, const float *q_norm, const float *k_norm, const InvFreq &inv_freq,
                                float eps, uint32_t *status, cudaStream_t stream, int sms);

// Where the output rows of a matmul go: rows [0, e0) to p0, [e0, e1) to p1,
// [e1, d) to p2, each as [B][segment length] (one segment: p0, e0 = e1 = d).
struct MmOut {
    float *p0, *p1, *p2;
    int e0, e1;
};
// The input of a fused one-token matmul, computed by every CTA into shared
// memory before its dot products:
//   PRO_RMS:    x = Q8_0(RMSNorm(a; weight w, eps))  (:281-291, then quantize)
//   PRO_SWIGLU: x = Q8_0(SwiGLU(a, b))               (:449-450, then :453)
// with the operations of rmsnorm_row_kernel and swiglu_v8_kernel, so the codes
// and scales are the ones those kernels store.
enum MmProKind { PRO_RMS = 1, PRO_SWIGLU = 2 };
struct MmPro {
    const float *a, *b, *w;
    float eps;
};
cudaError_t launch_matmul_q8_pro(MmProKind kind, const MmPro &pro, int n, const int8_t *wq, const float *ws, int d,
                                 const MmOut &out, cudaStream_t stream, int sms, const float *add);
// pdl: launched with programmatic stream serialization (may overlap the
// previous kernel in the stream, which must not read what this one writes).
cudaError_t launch_matmul_q8_seg(const int8_t *xq, const float *xs, int B, const int8_t *wq, const float *ws, int n,
                                 int d, const MmOut &out, cudaStream_t stream, int sms, const float *add = nullptr,
                                 bool pdl = false);
// out = W @ x for each token row; with `add`, out = add + W @ x (one rounding).
cudaError_t launch_matmul_q8(const int8_t *xq, const float *xs, int B, const int8_t *wq, const float *ws, int n,
                             int d, float *out, cudaStream_t stream, int sms, const float *add = nullptr);

// The same matmul for prefill-sized batches on the tcgen05 tensor cores
// (k_gemm.cu): B >= 128 token rows, n a multiple of 128.  Same bits.
bool matmul_q8_tc_supported(int B, int n, int d);
cudaError_t launch_matmul_q8_tc(const int8_t *xq, const float *xs, int B, const int8_t *wq, const float *ws, int n,
                                int d, float *out, uint32_t *status, cudaStream_t stream, int sms);

// One decode step's parameters, in device memory: the token, its position and
// RoPE's cos/sin(pos * freq_j) for j < 64 (head_dim 128), computed on the host.
struct StepParams {
    int32_t pos, token, pad0, pad1;
    float c[64], s[64];
};
// Writes v to *sp in stream order (a kernel: usable inside any stream capture).
cudaError_t launch_set_step(StepParams *sp, const StepParams &v, cudaStream_t stream);
// Attention of the step's token at sp->pos (head_dim 128), from the raw
// qkv = [q | k | v] rows of the Q|K|V matmul: QK-RMSNorm + RoPE of q and k
// (:361-393), k and v into the layer's cache rows at pos (kc / vc
// [seq_len][n_kv * 128]), scores, softmax and weighted values (:395-428;
// att [n_heads][seq_len] scratch), the output [n_heads][128] as Q8_0 codes xq
// and scales xs [n_heads * 2] (:431).  Two launches, the rotations inside the
// first, at every context length (above 16,384 positions the values launch
// recomputes each chunk's probabilities instead of keeping them all).
cudaError_t launch_attention_step(float *qkv, float *kc, float *vc, float *att, int8_t *xq, float *xs,
                                  const StepParams *sp, int n_heads, int n_kv, const float *qn, const float *kn,
                                  float eps, int seq_len, cudaStream_t stream, int sms);

// The attention of one token alone (qwen3_original.c:395-428, q already
// normalised and rotated, K/V rows 0..pos in the caches [..][kv_dim]): the
// scores into att [n_heads][att_stride] (att_stride > pos, scratch), the
// probabilities into probs (same shape, a different buffer; may be NULL) and
// the head outputs into xb [n_heads][128].  The decode step's two launches (scores over
// (head, chunk), then values over (head, half)); head_dim 128, any length.
cudaError_t launch_attention_rows(const float *q, const float *kc, const float *vc, float *att, float *probs, float *xb,
                                  int pos, int n_heads, int kv_dim, int kv_mul, int att_stride, cudaStream_t stream,
                                  int sms);

cudaError_t launch_swiglu(const void *hb, const void *hb2, q3cu_dtype dt, int64_t elems, void *out, int8_t *q,
                          float *s, uint32_t *status, cudaStream_t stream, int sms);

// `sched` is a pair of device counters, zero before the launch and zero
// again after it (the last CTA resets them); no two launches that may run at
// the same time share a pair.
constexpr int SMX_SCHED_WORDS = 2;
cudaError_t launch_softmax_rows(float *x, const int64_t *off, const int32_t *len, int64_t rows, uint32_t *sched,
                                uint32_t *status, cudaStream_t stream, int sms);

}  // namespace q3
