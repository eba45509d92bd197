/*
 * tsb.h — C ABI of libtsb.so, the B200 (sm_100a) verify-pass hot path of
 * mlx-tree-spec: the MLX 4-bit affine quantized matmul and tree-mask flash
 * attention over a long KV prefix, and the kernels either side of them (the
 * decoder layer's norms, rope and KV append, the tree commit of the KV
 * caches, GatedDeltaNet over tree nodes).
 *
 * Conventions (mirroring the reference's operator contract):
 *   - Every entry point returns an int status. TSB_OK on success.
 *     TSB_EUNSUPPORTED means "decline": the shape or format is one this library
 *     does not take, and the caller falls back, as the reference's kernels
 *     return None (mlx-tree-spec src/mlx_tree_spec/tree_flash.py:165-172,
 *     tree_verify.py:363-366). TSB_EINVAL is a contract violation (null or
 *     misaligned pointer, inconsistent sizes), as the reference's asserts
 *     (qmm_packed.py:113,227,375,705; tree_flash.py:113).
 *   - All pointers are device pointers unless stated otherwise. Inputs are
 *     read only. Nothing is allocated inside: scratch memory is passed by the
 *     caller as (ws, ws_bytes), sized by the matching *_workspace_bytes().
 *   - All work is enqueued on the caller's stream; calls are asynchronous and
 *     stateless, so concurrent calls on different streams are safe as long as
 *     their outputs and workspaces do not overlap.
 *   - bf16 tensors are passed as `const void*` holding IEEE bfloat16 values.
 */
#ifndef TSB_H
#define TSB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t / CUstream; NULL is the legacy default stream. */
typedef struct CUstream_st *tsb_stream_t;

enum {
  TSB_OK = 0,
  TSB_EUNSUPPORTED = 1, /* declined: caller falls back (tree_flash.py:165-172) */
  TSB_EINVAL = 2,       /* contract violation: bad pointer, size or alignment */
  TSB_ECUDA = 3,        /* CUDA runtime or launch error */
  TSB_ETIMEOUT = 4,     /* a bounded device-side wait gave up */
  TSB_EWORKSPACE = 5    /* workspace smaller than *_workspace_bytes() */
};

/* KV-cache formats read by tsb_tree_attn. */
enum {
  TSB_KV_BF16 = 0,       /* data bf16 [B,Hkv,cap,D]; scales = biases = NULL                */
  TSB_KV_MLX_Q8_G64 = 1, /* data uint32 [B,Hkv,cap,D/4] (4 codes, low byte first);
                            scales, biases bf16 [B,Hkv,cap,D/64]; value = s*q + b          */
  TSB_KV_REF_Q8_ROW = 2  /* data int8 [B,Hkv,cap,D]; scales float [B,Hkv,cap]; biases NULL;
                            value = q * s (mlx-tree-spec src/mlx_tree_spec/kv8.py:39-43)   */
};

/* Human-readable text of a status code (static storage). */
const char *tsb_strerror(int status);

/* Library version, (major << 16) | (minor << 8) | patch. */
int tsb_version(void);

/* Synchronizes `stream`, then returns the first failure any kernel recorded on
 * the device since the last reset: TSB_OK, or TSB_ETIMEOUT when a bounded
 * device-side wait (pipeline barrier) gave up instead of hanging. The kernel
 * that records it stops its work and returns, so the context stays usable.
 * reset != 0 clears the record. No counterpart in the reference (its Metal
 * kernels have no device-side waits). */
int tsb_device_status(tsb_stream_t stream, int reset);

/* ------------------------------------------------------------------------
 * Quantized matmul, MLX affine format, group 64, 4 bits.
 *
 * y[m, n] = sum_k x[m, k] * W[n, k],  W[n, k] = s[n, k/64] * q[n, k] + b[n, k/64]
 *
 * Replaces mx.quantized_matmul(x, w, scales, biases, transpose=True,
 * group_size=64, bits=4) as called by the reference's patched
 * nn.QuantizedLinear (mlx-tree-spec src/mlx_tree_spec/packed_linear.py:83-104,
 * call site 97) and its launchers (qmm_packed.py:270-293 nax_kernel,
 * 372-394 nax_multi_kernel, 529-557 _qmv_kernel, 701-725 prefill_kernel).
 *
 *   x      bf16 [M, K], row stride K
 *   w      uint32 [N, K/8]: word c of row n holds k = 8c..8c+7, element i in
 *          bits 4i..4i+3 (MLX layout, read directly, no repack)
 *   scales bf16 [N, K/64];  biases bf16 [N, K/64]
 *   y      bf16 [M, ldy] (ldy >= N; an N-shard may write into a wider buffer)
 * Requirements: M >= 1, N % 128 == 0, K % 64 == 0, ldy % 8 == 0; x, w, y
 * 16-byte aligned. Accumulation in float32. Declines (TSB_EUNSUPPORTED)
 * other N/K granularities.
 * Routing by M (the reference's packed_linear._call, packed_linear.py:10-13,
 * 83-104): M <= 2 a CUDA-core GEMV (x staged in shared memory; past its size
 * the verify kernel), M <= 128 the tcgen05 verify kernel, larger M the
 * tcgen05 prefill GEMM.
 *
 * Workspace (M <= 128, the verify path): tsb_qmm_workspace_bytes(M, N, K)
 * bytes, 256-byte aligned, computed for the current device. It holds
 * completion flags and float partials of row tiles shared between CTAs. It
 * must be zero-filled once before its first use (cudaMemset); every call
 * leaves it zero again. Do not share it with other work or with calls in
 * flight on another stream. Too small or NULL: TSB_EWORKSPACE. M > 128 (the
 * prefill GEMM) needs none (size 0).
 * ---------------------------------------------------------------------- */
size_t tsb_qmm_workspace_bytes(int M, int N, int K);
int tsb_qmm_w4g64(const void *x, const uint32_t *w, const void *scales, const void *biases, void *y,
                  int M, int N, int K, int ldy, void *ws, size_t ws_bytes, tsb_stream_t stream);

/* ------------------------------------------------------------------------
 * N-sharded quantized matmul with the output gathered over the GPUs of one
 * node inside the same kernel. The reference runs on one device; this is the
 * tensor-parallel form of tsb_qmm_w4g64 (the layer's full output on every GPU,
 * as an N-split matmul followed by an all-gather would leave it).
 *
 * Rank `rank` of `world` holds rows [rank*Ns, (rank+1)*Ns) of W (itself a
 * valid MLX-format weight of Ns rows) and computes columns [rank*Ns,
 * (rank+1)*Ns) of y. Its kernel stores that slice into every rank's y (peer
 * stores over NVLink), so when the call completes on a rank's stream, that
 * rank's y [M, ldy] holds all world*Ns columns.
 *   y[p]    rank p's output buffer, mapped into this process (peer memory);
 *           the same [M, ldy] layout on every rank
 *   sig[p]  rank p's signal block, mapped likewise: 2*world + 3 uint32,
 *           zero-filled once before the first call, then owned by these calls
 * Every rank makes the same sequence of calls with the same block (one block
 * per stream of calls); a rank that stops leaves its peers' calls to end in
 * TSB_ETIMEOUT (tsb_device_status). Before storing into a peer's y, a call
 * waits until that peer has started the same call, so work queued before it
 * on the peer's stream (readers of the old contents) has finished.
 * Any M: M <= 2 runs the GEMV, M <= 128 the verify kernel, larger M the
 * prefill GEMM, each storing its outputs into every rank's y as they complete
 * (the transfer overlaps the matmul). ldy >= world*Ns; workspace tsb_qmm_workspace_bytes(M, Ns, K)
 * (none past M = 128); other rules as tsb_qmm_w4g64.
 * ---------------------------------------------------------------------- */
#define TSB_MAX_GATHER_RANKS 8
typedef struct {
  int world, rank;
  void *y[TSB_MAX_GATHER_RANKS];
  uint32_t *sig[TSB_MAX_GATHER_RANKS];
} tsb_gather_t;
int tsb_qmm_w4g64_gather(const void *x, const uint32_t *w, const void *scales, const void *biases, int M, int Ns,
                         int K, int ldy, const tsb_gather_t *g, void *ws, size_t ws_bytes, tsb_stream_t stream);

/* Bit-exact dequantization: out[n, k] = bf16_rne(fmaf(q, s, b)) as bf16 [N, K].
 * Reference rule: `T(float(q) * s + b)` in qmm_packed.py:200,348,635.
 * Requirements: K % 64 == 0. */
int tsb_dequant_w4g64(const uint32_t *w, const void *scales, const void *biases, void *out,
                      int N, int K, tsb_stream_t stream);

/* ------------------------------------------------------------------------
 * Tree masks.
 *
 * parents int32 [B, T]: parent of each node (-1 for a root; otherwise an
 * earlier node). bits uint64 [B, T]: bit j of node i set iff j is i or one of
 * its ancestors. depth int32 [B, T] (nullable): 0 for roots. Replaces
 * Tree.__init__/ancestor_bits (mlx-tree-spec src/mlx_tree_spec/tree_verify.py:
 * 66-121, tree_flash.py:146-148), extended to forests. T <= 64. A parent that
 * is neither -1 nor an earlier node yields bits = 0 and depth = -1 for that
 * node (the reference asserts, tree_verify.py:71).
 * ---------------------------------------------------------------------- */
int tsb_tree_ancestor_bits(const int32_t *parents, int B, int T, uint64_t *bits, int32_t *depth,
                           tsb_stream_t stream);

/* Element types of an attention mask read by tsb_tree_mask_bits. */
enum {
  TSB_MASK_BOOL = 0, /* uint8: nonzero = visible                                  */
  TSB_MASK_BF16 = 1, /* additive bf16: +-0 = visible, -inf = hidden               */
  TSB_MASK_F16 = 2,  /* additive fp16: +-0 = visible, -inf = hidden               */
  TSB_MASK_F32 = 3   /* additive float: +-0 = visible, -inf = hidden              */
};

/* An attention mask in the form SDPA takes -> the bit form tsb_tree_attn
 * takes: the inverse of Tree.mask (mlx-tree-spec src/mlx_tree_spec/
 * tree_verify.py:131-139, where(anc, 0, -inf) after `offset` zero columns),
 * for callers that hold the reference's additive mask (the mlx-lm SDPA hook,
 * long_attention.py:69-88; the SDPA fallback, tree_verify.py:363-366).
 *
 *   mask  rows x L elements of mask_dtype, row r at element r * row_stride
 *   bits  uint64 [rows]: bit j set iff column L - tail + j is visible
 *   bad   int32 [1], set to the number of rows the bit form cannot express:
 *         a hidden column before the last `tail`, or an additive value that
 *         is neither +-0 nor -inf (a bias, +inf, NaN). Such a row's bits are
 *         meaningless; the caller keeps the mask (its own SDPA).
 * Requirements: rows >= 1, 0 <= tail <= L <= row_stride, tail <= 64. */
int tsb_tree_mask_bits(const void *mask, int mask_dtype, int rows, long long L, long long row_stride, int tail,
                       uint64_t *bits, int32_t *bad, tsb_stream_t stream);

/* ------------------------------------------------------------------------
 * Tree-mask flash attention (split-KV flash decoding with fused combine).
 *
 * out[b, h, t, :] = softmax_j(scale * q[b,h,t] . k[b,h/G,j] over visible j) . v
 * with G = Hq / Hkv. Row j (0 <= j < n_kv) is visible to node t iff
 * j < n_kv - tail, or bit (j - (n_kv - tail)) of the node's mask is set.
 * The mask comes from `parents` (int32 [B, T], tail = T: the nodes' own K/V
 * are the cache's last T valid rows) when non-NULL, computed inside the
 * kernel; otherwise from `bits` (uint64 [B, T], any tail <= 64; tail 0 makes
 * every row visible). Replaces tree_flash(queries, cache, scale, bits, tail,
 * stats) (mlx-tree-spec src/mlx_tree_spec/tree_flash.py:151-196) and the q8
 * path kv8.attention (kv8.py:162-188), without its bsz == 1 / n <= 16 /
 * tail <= 64-only limits except tail <= 64.
 *
 *   q        bf16 [B, Hq, T, D]
 *   k, v     per kv_format (see TSB_KV_*), kv_capacity rows per (b, head)
 *   out      bf16 [B, Hq, T, D]
 *   lse      float [B, Hq, T] (nullable): natural-log sum of exp of the
 *            visible scaled scores (-inf for a node that sees nothing), the
 *            statistic that lets more keys be merged in later (the block
 *            max/sum of tree_flash(stats=True) collapsed to one block).
 * Requirements: D == 256, Hq % Hkv == 0, 1 <= T <= 64, n_kv <= kv_capacity.
 * ---------------------------------------------------------------------- */
size_t tsb_tree_attn_workspace_bytes(int B, int T, int Hq, int Hkv, int D, int n_kv, int kv_format);
int tsb_tree_attn(const void *q,
                  const void *k, const void *k_scales, const void *k_biases,
                  const void *v, const void *v_scales, const void *v_biases,
                  int kv_format, const int32_t *parents, const uint64_t *bits,
                  int B, int T, int Hq, int Hkv, int D, int n_kv, int tail, int kv_capacity,
                  float scale, void *out, float *lse, void *ws, size_t ws_bytes, tsb_stream_t stream);

/* Allocation-free tsb_tree_attn, for callers that cannot pass a workspace
 * (a host whose device memory belongs to a pool allocator it cannot call from
 * the decode loop, an FFI binding without a device allocator, a serving loop
 * that forbids allocation). Same arguments and result as tsb_tree_attn minus
 * (ws, ws_bytes). The split-KV scratch is a fixed 16 MiB array inside the
 * library, reserved on each GPU that loads it and held until the process
 * exits; a call whose tsb_tree_attn_workspace_bytes() exceeds 16 MiB returns
 * TSB_EWORKSPACE without launching anything (use tsb_tree_attn with a
 * workspace then). The first call on each device looks up the array's device
 * address: make it before any stream capture. All calls on a device share the
 * array, so calls whose GPU work overlaps race: serialize them. No counterpart
 * in the reference (its MLX kernels allocate their outputs per call). */
int tsb_tree_attn_noalloc(const void *q,
                          const void *k, const void *k_scales, const void *k_biases,
                          const void *v, const void *v_scales, const void *v_biases,
                          int kv_format, const int32_t *parents, const uint64_t *bits,
                          int B, int T, int Hq, int Hkv, int D, int n_kv, int tail, int kv_capacity,
                          float scale, void *out, float *lse, tsb_stream_t stream);

/* ------------------------------------------------------------------------
 * Verify-step decoder layer: the kernels around the qmm and tree attention
 * (mlx-tree-spec src/mlx_tree_spec/tree_verify.py:311-367 batch_attention /
 * _attn_core, 414-447 batch_forward; fused_ops.py:107-154 add_rms_norm). All
 * tensors bf16, row-major, 16-byte aligned; launches on `stream`.
 * ---------------------------------------------------------------------- */

/* Residual add + RMS norm (fused_ops.py:107-154): h = bf16(x + r),
 * n = bf16(w * bf16(h * rsqrt(mean(h^2) + eps))) per row of D values. r NULL:
 * the plain norm of x (nn.RMSNorm); h_out may be NULL. D % 8 == 0, D <= 16384. */
int tsb_add_rms_norm(const void *x, const void *r, const void *w, void *h_out, void *n_out, int rows, int D,
                     float eps, tsb_stream_t stream);

/* Per-node q/k/v preparation for gated-q tree attention (tree_verify.py:
 * 316-323, 331-362). qkv [B*T, ld]: per query head h the 2*D columns
 * [h*2D, h*2D + D) query and [h*2D + D, (h+1)*2D) gate, then Hkv key heads,
 * then Hkv value heads (D each). Queries and keys get the per-head RMS norm
 * (q_norm / k_norm weights [D]) and mx.fast.rope (non-traditional, the first
 * rope_dims dims, base, scale) at positions[b*T + t]; queries go to q_out
 * [B, Hq, T, D]; keys and values are appended to the caches at rows
 * offsets[b] + t (capacity rows per (request, head)) in kv_format, quantized on
 * append for the 8-bit formats (TSB_KV_REF_Q8_ROW as kv8.py:39-43, MLX g64 as
 * this library's quantizer). D == 256; rope_dims % 16 == 0. */
int tsb_qkv_prep(const void *qkv, int ld, int B, int T, int Hq, int Hkv, int D, const void *q_norm,
                 const void *k_norm, float eps, const int32_t *positions, int rope_dims, float rope_base,
                 float rope_scale, void *q_out, int kv_format, void *k, void *k_scales, void *k_biases, void *v,
                 void *v_scales, void *v_biases, int kv_capacity, const int32_t *offsets, tsb_stream_t stream);

/* y [B*T, Hq*D] = attention out [B, Hq, T, D] * sigmoid(gate), the gate read
 * from qkv as laid out above (tree_verify.py:327: o_proj's input). D == 256. */
int tsb_attn_gate(const void *attn_out, const void *qkv, int ld, void *y, int B, int T, int Hq, int D,
                  tsb_stream_t stream);

/* SwiGLU: y [M, I] = silu(g) * u for gate_up [M, 2I] = [g | u] (the MLP's
 * fused gate and up projections). I % 8 == 0. */
int tsb_swiglu(const void *gate_up, void *y, int M, int I, tsb_stream_t stream);

/* Tree commit (tree_verify.py:487-496 _keep_kv; kv8.py:143-148 take_rows):
 * for request b, rows offsets[b] + nodes[b*max_keep + i], i < n_keep[b], of
 * every KV head's K and V (and their scales / biases in the 8-bit formats)
 * move to rows offsets[b] + i. Rows are read before any is written, so a path
 * may overlap its destination. offsets, nodes, n_keep are HOST arrays (copied
 * into the launch's parameters; nothing is allocated or copied to the
 * device). Caches laid out as for tsb_tree_attn. D == 256, B <= 8,
 * max_keep <= 64, every node < 64 (the tree width bound); node and
 * destination rows must lie below kv_capacity (else TSB_EINVAL). */
int tsb_kv_commit(int kv_format, void *k, void *k_scales, void *k_biases, void *v, void *v_scales, void *v_biases,
                  int B, int Hkv, int D, int kv_capacity, const int32_t *offsets, const int32_t *nodes,
                  const int32_t *n_keep, int max_keep, tsb_stream_t stream);

/* The same commit for every layer's cache in one launch (tree_verify.py:
 * 499-516 commit loops over the layers): k, v, k_scales ... are HOST arrays
 * of `layers` device pointers (the scale / bias arrays NULL where the format
 * has none), all caches of one format and shape. layers <= 48. */
int tsb_kv_commit_layers(int kv_format, int layers, void *const *k, void *const *k_scales, void *const *k_biases,
                         void *const *v, void *const *v_scales, void *const *v_biases, int B, int Hkv, int D,
                         int kv_capacity, const int32_t *offsets, const int32_t *nodes, const int32_t *n_keep,
                         int max_keep, tsb_stream_t stream);

/* ------------------------------------------------------------------------
 * GatedDeltaNet over tree nodes (the hybrid model's linear-attention layers;
 * mlx-tree-spec tree_verify.py:149-238, fused_ops.py:28-104, 157-226). One
 * request's n tree nodes per call. Dk = Dv = 128, Hv % Hk == 0 (else
 * TSB_EUNSUPPORTED). bf16 tensors row-major, 8-byte aligned; state float32
 * [Hv, Dv, Dk], 16-byte aligned. Node-major layouts: q, k [n, Hk, Dk];
 * v, y [n, Hv, Dv]; g, beta, a, b [n, Hv]. C = (2*Hk + Hv) * 128.
 * ---------------------------------------------------------------------- */

/* gdn_prep (fused_ops.py:28-104): per node the causal conv (kernel 4) over
 * rows conv_idx[node*4 + 0..3] of concat(conv_state [3, C], qkv [n, C]) with
 * weights conv_w [C, 4], bf16, silu, bf16; v = that; q, k = per-head RMS norm
 * (eps 1e-6, bf16) times 1/Dk and Dk^-1/2; beta = sigmoid(b) (bf16);
 * g = exp(-exp(a_log) * bf16(softplus(bf16(a + dt_bias)))) (float32).
 * a_log, dt_bias float32 [Hv]. conv_idx is a device array (n x 4). */
int tsb_gdn_prep(const void *qkv, const void *conv_state, const int32_t *conv_idx, const void *conv_w, const void *a,
                 const void *b, const float *a_log, const float *dt_bias, void *q, void *k, void *v, float *g,
                 void *beta, int n, int Hk, int Dk, int Hv, int Dv, tsb_stream_t stream);

/* tree_gated_delta (tree_verify.py:149-238): y[node] = the gated delta
 * recurrence's output at `node` along its root path, from `state` (the
 * committed state, not modified). Walks: device arrays paths, sibs
 * [rows, lmax] (node indices, -1 past a walk's end / no sibling) and owner [n]
 * (the walk that writes each node's output); every node must appear in some
 * walk as a path node or a sibling. Out-of-range indices end a walk. */
int tsb_tree_gated_delta(const void *q, const void *k, const void *v, const float *g, const void *beta,
                         const float *state, const int32_t *paths, const int32_t *sibs, const int32_t *owner, int rows,
                         int lmax, int n, int Hk, int Dk, int Hv, int Dv, void *y, tsb_stream_t stream);

/* gdn_commit (fused_ops.py:157-226): state_out = the state after the accepted
 * path nodes[0..n_keep) (a HOST int32 array, each < min(n, 64)) replayed from
 * state_in (state_out may equal state_in); conv_out [3, C] = rows
 * conv_idx[last*4 + 1..3] of concat(conv_state, qkv), last = nodes[n_keep-1].
 * conv_out must not overlap conv_state (TSB_EINVAL): other CTAs may still be
 * reading conv_state while it is written. */
int tsb_gdn_commit(const void *k, const void *v, const float *g, const void *beta, const float *state_in,
                   const void *conv_state, const void *qkv, const int32_t *conv_idx, const int32_t *nodes, int n_keep,
                   int n, int Hk, int Dk, int Hv, int Dv, float *state_out, void *conv_out, tsb_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* TSB_H */
