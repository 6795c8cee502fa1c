/* hsg.h -- C ABI of the HS-Guard B200 streaming engine (libhsg.so, sm_100a).
 *
 * The engine replaces the reference's slot engine object, i.e. the construction
 *     self.engine = SlotStreamEngineV8(model, max_slots, ...)          src/hs_guard/runtime.py:157
 * and its per-tick call
 *     self.engine.step(requests)[role]                                 src/hs_guard/runtime.py:172
 * whose device work is SlotStreamEngineV7._run_arrays (src/hs_guard/engine/slot_engine_v7.py:117-136):
 * copy the packed tick to the GPU, replay the tick's CUDA graph, copy the class probabilities back.
 * The Python host (hs_guard_b200.runtime.StreamingGuard) keeps the reference's validation, token splitting,
 * bucket choice, pack_inputs layout and per-slot lengths, and calls these functions.
 *
 * Conventions: every function returns HSG_OK (0) or a negative HSG_ERR_* code; hsg_last_error() then describes
 * the failure (thread-local string). Nothing throws across the ABI. "device pointer" arguments are CUDA global
 * memory on the engine's device; "host pointer" arguments are ordinary (ideally pinned) host memory.
 * An engine is used by one host thread at a time (the reference's single owner thread, examples/demo/batching.py:20).
 */
#ifndef HSG_H
#define HSG_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HSG_OK 0
#define HSG_ERR_INVALID (-1)     /* invalid argument (Python: ValueError) */
#define HSG_ERR_CUDA (-2)        /* CUDA runtime failure (RuntimeError) */
#define HSG_ERR_DEVICE (-3)      /* a kernel reported a bounded-wait timeout or an out-of-range index */
#define HSG_ERR_UNSUPPORTED (-4) /* architecture or device the kernels are not built for */

#define HSG_N_LAYERS 24

/* Architecture (reference: transformers Qwen3_5TextConfig as built by load_model, runtime.py:103-113, and the
 * window of metadata['window_tokens'], runtime.py:117). hsg_create rejects anything but the HS-Guard backbone:
 * 1024 hidden, 3584 MLP, 24 layers with attention every 4th, 16 GDN heads of 128, 8/2 attention heads of 256,
 * 64 rotary dims, 512-token window, two 512-wide 3-class role heads. */
typedef struct hsg_config {
  int32_t hidden, intermediate, n_layers, full_attn_interval;
  int32_t gdn_heads, gdn_head_dim, conv_kernel;
  int32_t attn_heads, kv_heads, attn_head_dim, rotary_dim;
  int32_t vocab, window, head_hidden, n_classes, n_roles;
  float rms_eps, head_ln_eps;
} hsg_config;

/* Per-layer weights in the engine layout (device pointers, borrowed: they must outlive the engine).
 * GDN layers use w_in = [in_proj_qkv | in_proj_z | in_proj_b | in_proj_a | zero pad] (8320 x 1024 bf16) and
 * conv_w / A_log / dt_bias / gnorm_w; attention layers use w_in = [q_proj | k_proj | v_proj] (5120 x 1024 bf16)
 * and q_norm / k_norm. w_gu interleaves gate_proj and up_proj row by row (row 2f = gate f, row 2f+1 = up f;
 * 7168 x 1024 bf16). All RMSNorm weights are passed as fp32 (1 + w); gnorm_w is the gated norm's plain w. */
typedef struct hsg_layer_weights {
  const void* w_in;
  const void* w_out;     /* out_proj / o_proj, 1024 x 2048 bf16 */
  const void* w_gu;
  const void* w_down;    /* 1024 x 3584 bf16 */
  const float* norm_in;  /* input_layernorm, 1 + w */
  const float* norm_post;/* post_attention_layernorm, 1 + w */
  const float* conv_w;   /* [6144][4] fp32 */
  const float* A_log;    /* [16] */
  const float* dt_bias;  /* [16] */
  const float* gnorm_w;  /* [128] */
  const float* q_norm;   /* [256] 1 + w */
  const float* k_norm;   /* [256] 1 + w */
} hsg_layer_weights;

typedef struct hsg_weights {
  const void* embed;        /* [vocab][1024] bf16 */
  const float* final_norm;  /* [1024] 1 + w */
  const float* inv_freq;    /* [32] RoPE inverse frequencies (fp32, as transformers computes them) */
  hsg_layer_weights layers[HSG_N_LAYERS];
  const void* head_w1;      /* [n_roles*512][1024] bf16, roles in order (user, assistant) */
  const float* head_b1;     /* [n_roles*512] */
  const float* head_ln_w;   /* [n_roles*512] LayerNorm weight */
  const float* head_ln_b;   /* [n_roles*512] LayerNorm bias */
  const float* head_w2;     /* [n_roles][3][512] fp32 */
  const float* head_b2;     /* [n_roles][3] */
} hsg_weights;

typedef struct hsg_engine hsg_engine;

/* Device pointers of the engine's state pools (for snapshots, tests and diagnostics). S = max_slots; slot S is
 * the scratch slot padded rows use (reference engine/bucketed_engine.py:37-42). */
#define HSG_STATE_F32 0
#define HSG_STATE_F16 1
typedef struct hsg_pools {
  void* rec;           /* [n_gdn=18][S+1][16][128][128] gated-delta-rule state, element type rec_dtype */
  float* conv;         /* [18][S+1][3][6144] fp32 causal-conv history */
  void* ring_k;        /* [n_attn=6][S+1][2][513][256] fp16 */
  void* ring_v;        /* same */
  int64_t* ring_pos;   /* [S+1][513], -1 = empty; column 512 is scratch */
  int32_t max_slots, n_gdn, n_attn;
  int32_t rec_dtype;   /* HSG_STATE_F16 (default) or HSG_STATE_F32 */
} hsg_pools;

/* Create an engine for slots 0..max_slots-1 on CUDA device `device` (replaces SlotStreamEngineV8.__init__,
 * engine/slot_engine_v8.py:179-195, with pools of engine/bucketed_engine.py:37-42). The recurrent state is stored
 * as fp16, the state_dtype StreamingGuard gives the reference engine (runtime.py:157); HSG_FLAG_STATE_F32 keeps it in
 * fp32 instead. HSG_FLAG_BF16_ACT feeds the GEMMs the bf16 activation only (the reference's autocast precision)
 * instead of the hi/lo pair. */
#define HSG_FLAG_BF16_ACT 1
#define HSG_FLAG_STATE_F32 2
int hsg_create(const hsg_config* cfg, const hsg_weights* weights, int max_slots, int device, int flags,
               hsg_engine** out);
int hsg_destroy(hsg_engine* eng);

/* One tick (SlotStreamEngineV7._run_arrays, slot_engine_v7.py:117-136). `packed` (host pointer) holds
 * nb*lb + 3*nb int64 in the pack_inputs layout (slot_engine_v7.py:7-25): ids [nb][lb] | lens | slots | starts.
 * Writes out_probs (host pointer) [2 roles][nb][lb][3] fp32 softmax probabilities (safe, unsafe, controversial)
 * and returns after the copy back, like the reference's stream synchronize. Rows with lens 0 must use slot
 * max_slots; slots of rows with lens > 0 must be distinct. */
int hsg_step(hsg_engine* eng, const int64_t* packed, int nb, int lb, float* out_probs);

/* The same tick split in three asynchronous parts on the engine's stream, for callers that overlap host work or
 * keep inputs on the device: stage (host -> device copy of `packed`), launch (graph replay; `packed_dev` is a
 * device copy of the packed tick or NULL for the staged one) and fetch (device -> host copy of the probabilities,
 * stream synchronize and error check). */
int hsg_stage(hsg_engine* eng, const int64_t* packed, int nb, int lb);
int hsg_launch(hsg_engine* eng, const int64_t* packed_dev, int nb, int lb);
int hsg_fetch(hsg_engine* eng, int nb, int lb, float* out_probs);
int hsg_synchronize(hsg_engine* eng);
void* hsg_stream(hsg_engine* eng); /* the engine's cudaStream_t */

/* Zero every pool and mark every ring empty (BucketedStreamEngine.reset, bucketed_engine.py:51-55). */
int hsg_reset_all(hsg_engine* eng);
/* Per-slot state management (the demo's slot checkpoint/restore by tensor slicing, examples/demo/runtime_v10.py:98-111):
 * reset one slot, or copy its state (all pools) to / from a device buffer of hsg_slot_state_bytes() bytes. */
int hsg_reset_slot(hsg_engine* eng, int slot);
size_t hsg_slot_state_bytes(const hsg_engine* eng);
int hsg_snapshot_slot(hsg_engine* eng, int slot, void* dst_device);
int hsg_restore_slot(hsg_engine* eng, int slot, const void* src_device);
int hsg_get_pools(const hsg_engine* eng, hsg_pools* out);

/* Run one tick eagerly (no graph) timing each kernel with CUDA events; kernel_ms[i] / launches[i] accumulate per
 * kernel class i (HSG_PROF_* below). Used by the benchmark for the roofline of the dominant kernel. */
enum {
  HSG_PROF_EMBED = 0, HSG_PROF_GEMM_IN, HSG_PROF_GDN, HSG_PROF_ATTN_PREP, HSG_PROF_RING_ATTN, HSG_PROF_RING_APPEND,
  HSG_PROF_GEMM_OUT, HSG_PROF_NORM, HSG_PROF_GEMM_GU, HSG_PROF_GEMM_DOWN, HSG_PROF_HEAD_GEMM, HSG_PROF_HEAD,
  HSG_PROF_COMMIT, HSG_PROF_N
};
int hsg_profile_step(hsg_engine* eng, const int64_t* packed, int nb, int lb, float* out_probs, float* kernel_ms,
                     int* launches);
/* Kernel launches one tick of shape (nb, lb) makes (the graph's kernel nodes). */
int hsg_launches_per_step(const hsg_engine* eng, int nb, int lb);

/* ---- isolated kernels (stream = cudaStream_t or NULL for the default stream; err = device int, 0 on entry) ---- */

/* Gated-delta-rule slot step with the contract of the reference's gdn_slot_v8 (engine/fused_kernels.py:197-211):
 * packed [n][lb][6144] bf16 (q | k | v after conv+SiLU), a, b [n][lb][16] fp32 raw projections, A_log, dt_bias [16],
 * state [max_slots+1][16][128][128] (HSG_STATE_F32 or HSG_STATE_F16) updated in place at rows slots[i] with
 * lens[i] > 0; writes o [n][lb][16][128] fp32 (zeros at padded positions). All device pointers. fp32 state with
 * n <= 32 rows runs one CTA per 32-column slice of each (row, head) state (a small batch in one wave); other shapes
 * the engine's persistent kernels. */
int hsg_gdn_step(const void* packed, const float* a, const float* b, const float* A_log, const float* dt_bias,
                 void* state, int state_dtype, const int64_t* slots, const int64_t* lens, int n, int lb,
                 int max_slots, float* o, int* err, void* stream);

/* Ring-window GQA attention with the contract of the reference's ring_attention (engine/ring_attention_kernel.py:
 * 164-178): q [n][2][4*lb][256] fp32, ring_k/v [max_slots+1][2][513][256] fp16, new_k/v [n][2][lb][256] fp16,
 * ring_pos [max_slots+1][513] int64, slots/starts/lens [n] int64; writes out [n][2][4*lb][256] fp32. With
 * write_ring = 1 (lb == 1 only) the new key/value are also stored at column starts % 512, as the engine does. */
int hsg_ring_attention(const float* q, void* ring_k, void* ring_v, const void* new_k, const void* new_v,
                       const int64_t* ring_pos, const int64_t* slots, const int64_t* starts, const int64_t* lens,
                       int n, int lb, int max_slots, float scale, float* out, int write_ring, int* err, void* stream);

/* The engine's tensor-core GEMM on its own: y[m][n] (+)= sum_k x[m][k] w[n][k] with x given as bf16 hi (and
 * optional lo) [m_alloc][k], w bf16 [n][k]; mode 0 store, 1 add into y (TMA bulk reduce-add, with `splits` K
 * splits), 2 SiLU-mul of row-interleaved (gate, up) pairs into act_hi/act_lo [m][n/2]. n % 128 == 0, k % 64 == 0,
 * 16-byte aligned pointers; y has row stride n. */
int hsg_gemm(const void* w, int n, int k, const void* x_hi, const void* x_lo, int m, int m_alloc, float* y,
             void* act_hi, void* act_lo, int mode, int splits, int* err, void* stream);

/* hsg_gemm for fp32 activations x [m][k] (16-byte aligned) that allocates nothing: the bf16 (hi, lo) operand pair
 * is built in a fixed scratch area compiled into the library (HSG_NOALLOC_MAX_ELEMS elements of each half,
 * 8 MiB in all, one per device, held until the process exits), then the same tensor-core GEMM runs on it. Other
 * arguments and results are as in hsg_gemm. m * k above HSG_NOALLOC_MAX_ELEMS is rejected with HSG_ERR_INVALID.
 * The first call on a device (in each CUDA context of it) does a one-time set-up: it resolves the scratch area's
 * address (cudaGetSymbolAddress) and sets the GEMM kernels' shared-memory limit. With lazy module loading that first
 * call is also where the runtime may load the library's device code and place the area, so it is the one call that
 * can allocate; make it before capturing the stream into a graph. Later calls allocate nothing. Calls on one device
 * share the scratch area: calls on the same stream are ordered, calls that overlap in time on different streams
 * race. No counterpart in the reference (its GEMMs allocate through PyTorch). */
#define HSG_NOALLOC_MAX_ELEMS (1 << 21)
int hsg_gemm_f32_noalloc(const void* w, int n, int k, const float* x, int m, float* y, void* act_hi, void* act_lo,
                         int mode, int splits, int* err, void* stream);

/* Diagnostic of the failure path every kernel relies on (no counterpart in the reference): one thread on `device`
 * waits, with the kernels' own bounded wait, on a barrier that nothing completes. The wait gives up after its limit
 * (2 s) and records ERR_TIMEOUT_TMA in an error word, as a stalled pipeline in the engine would; the call returns
 * HSG_OK once that word has been read back with the timeout recorded (seconds = how long it took), HSG_ERR_DEVICE if
 * the wait ended without recording it. The GPU stays usable. */
int hsg_check_bounded_wait(int device, double* seconds);

const char* hsg_last_error(void);
const char* hsg_version(void);

#ifdef __cplusplus
}
#endif
#endif /* HSG_H */
