/* hive_b200 — C ABI of the B200-native batch-1 W4A8 Qwen3 decode library.
 *
 * Drop-in for HIVE Limited's driver layer: engine/cudrv.py (ctypes over libcuda plus the
 * PTX loader) and the eleven PTX entry points engine/limited.py launches through it.
 * Each declaration names the reference interface it replaces.
 *
 * Conventions
 *   - Every function returns an int status: HV_OK (0) on success, a CUDA runtime error
 *     code (1..999) when a CUDA call failed, or an HV_E_* code (>= 1000). The message of
 *     the most recent failure on the calling thread is read with hv_last_error(). The
 *     library never calls exit() or abort().
 *   - Device pointers are plain pointers into memory from hv_alloc() (or any CUDA
 *     allocation on the current device); sizes are element or byte counts as named.
 *   - `stream` is a cudaStream_t passed as void*; NULL is the legacy default stream
 *     (the stream the reference launches on outside graph capture).
 *   - Threads: calls act on the device current on the calling thread; a thread that did
 *     not create the engine binds it first with hv_set_device() (engine/limited.py:430-436
 *     bind_thread, engine/cudrv.py:124-132 set_current).
 *   - Device-resident scalars (token, position, step) are int32 device pointers, as in
 *     the reference (engine/limited.py:336-343).
 */
#ifndef HIVE_B200_H
#define HIVE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HV_ABI_VERSION 3

#define HV_OK 0
#define HV_E_INVALID 1001      /* bad argument (null pointer, size, alignment) */
#define HV_E_UNSUPPORTED 1002  /* shape outside what the kernels implement */
#define HV_E_NODEVICE 1003     /* no CUDA device */
#define HV_E_TIMEOUT 1004      /* a bounded device-side wait ran out (see hv_step_status) */
#define HV_E_CAPTURE 1005      /* operation not allowed while the stream is being captured */
#define HV_E_COMM 1006         /* collective / peer setup failed */

/* ---- library ------------------------------------------------------------------- */

/* ABI version of the loaded library (HV_ABI_VERSION). Replaces the kernel manifest
 * check of engine/limited.py:218-235 together with hv_kernel_list(). */
int hv_version(void);
/* Comma-separated names of the device entry points compiled into this library. */
int hv_kernel_list(char* buf, size_t len);
/* Copies the calling thread's most recent error message (NUL-terminated). */
int hv_last_error(char* buf, size_t len);

/* ---- device and context (engine/cudrv.py:73-135) -------------------------------- */

int hv_init(void);                                            /* cudrv.init          :73-74  */
int hv_device_count(int* n);
int hv_set_device(int dev);                                   /* cudrv.set_current   :124-132 */
int hv_get_device(int* dev);                                  /* cudrv.device        :77-80  */
int hv_device_name(int dev, char* buf, int len);              /* cudrv.device_name   :83-86  */
int hv_compute_capability(int dev, int* major, int* minor);   /* cudrv.compute_capability :106-114 */
int hv_device_attribute(int dev, int attr, int* value);       /* cudrv.device_attribute :99-103 (CUdevice_attribute numbering) */
int hv_driver_version(int* version);                          /* cudrv.driver_version :89-96 */
int hv_mem_info(size_t* free_bytes, size_t* total_bytes);     /* cudrv.mem_info      :139-143 */
int hv_synchronize(void);                                     /* cudrv.synchronize   :135-136 */

/* ---- memory (engine/cudrv.py:148-172) -------------------------------------------- */

/* Sizes are rounded up to 256 bytes, so bulk prefetches that round a range outwards to
 * 16 bytes stay inside the allocation. */
int hv_alloc(void** ptr, size_t nbytes);                      /* cudrv.alloc   :148-151 */
int hv_free(void* ptr);                                       /* cudrv.free    :154-155 */
int hv_upload(void* dst, const void* host_src, size_t nbytes);    /* cudrv.upload  :158-161 */
int hv_download(void* host_dst, const void* src, size_t nbytes);  /* cudrv.download :164-167 */
int hv_memset(void* ptr, int value, size_t nbytes);           /* cudrv.memset8 :170-173 */
int hv_host_alloc(void** ptr, size_t nbytes);                 /* pinned host memory */
int hv_host_free(void* ptr);
int hv_upload_async(void* dst, const void* host_src, size_t nbytes, void* stream);
int hv_download_async(void* host_dst, const void* src, size_t nbytes, void* stream);
int hv_copy_async(void* dst, const void* src, size_t nbytes, void* stream);

/* Cross-process device memory (CUDA IPC) for the sharded step's peer buffers: a
 * 64-byte handle of an allocation made by this process, and the mapping of another
 * process's handle into this one (peer access over NVLink enabled on first use). No
 * counterpart in the reference (it has no multi-GPU path). */
#define HV_IPC_HANDLE_BYTES 64
int hv_ipc_handle(const void* dev_ptr, void* handle_out);
int hv_ipc_open(const void* handle, void** dev_ptr);
int hv_ipc_close(void* dev_ptr);

/* The column-parallel layout's all-gather as a collective (NCCL over NVLink/NVSwitch),
 * for callers outside the fused step (which exchanges its slices itself): every rank
 * contributes `bytes` and every rank receives all contributions, rank after rank. No
 * counterpart in the reference (it has no multi-GPU path); the collective that a sharded
 * deployment of its GEMV (engine/limited.py:364-372) needs between layers.
 *   hv_comm_init       one process driving ndev GPUs (devs[i], rank i)
 *   hv_comm_unique_id  an id (HV_COMM_ID_BYTES) made on one rank, handed to every rank
 *   hv_comm_init_rank  one process per GPU: rank `rank` of `nranks` on device `dev`
 *   hv_allgather       send[i] / recv[i] / streams[i] for each device the process drives
 *                      (recv[i] holds nranks * bytes); asynchronous on the streams
 *   hv_comm_size       ranks of the communicator, devices this process drives
 *   hv_comm_destroy    frees the communicator (NULL is a no-op) */
#define HV_COMM_ID_BYTES 128
typedef struct hv_comm hv_comm;
int hv_comm_init(int ndev, const int* devs, hv_comm** out);
int hv_comm_unique_id(void* id_out);
int hv_comm_init_rank(int nranks, int rank, const void* id, int dev, hv_comm** out);
int hv_allgather(hv_comm* comm, const void* const* send, void* const* recv, size_t bytes,
                 void* const* streams);
int hv_comm_size(const hv_comm* comm, int* nranks, int* ndev);
int hv_comm_destroy(hv_comm* comm);

/* ---- streams, graphs, events (engine/cudrv.py:226-266) --------------------------- */

int hv_stream_create(void** stream);                          /* cudrv.stream_create :226-230 */
int hv_stream_destroy(void* stream);
int hv_stream_synchronize(void* stream);                      /* cudrv.stream_synchronize :233-234 */
int hv_capture_begin(void* stream);                           /* cudrv.capture_begin :237-240 */
int hv_capture_end(void* stream, void** graph);               /* cudrv.capture_end   :243-247 */
int hv_graph_instantiate(void* graph, void** exec);           /* cudrv.graph_instantiate :250-256 */
int hv_graph_launch(void* exec, void* stream);                /* cudrv.graph_launch :259-261 */
int hv_graph_destroy(void* graph, void* exec);                /* cudrv.graph_destroy :264-270 */
int hv_event_create(void** event);
int hv_event_destroy(void* event);
int hv_event_record(void* event, void* stream);
int hv_event_elapsed_ms(void* start, void* end, float* ms);

/* ---- kernels: one per reference PTX entry point (engine/limited.py:173-181) ------ */

/* quant_a8s (k_qa8s.ptx; launch engine/limited.py:368-369). Per-32 int8 activation
 * quantisation of src[nb*32]: a8[nb*32] int8; sa[0..nb) f32 scales and sa[nb..2nb) the
 * int32 block sums stored bit-for-bit in the same f32 array. */
int hv_qa8s(const float* src, int8_t* a8, float* sa, int nb, void* stream);

/* gemv_wpo_a4 (k_a4gv.ptx; launch engine/limited.py:370-372). dst[n] f32 for an
 * int4 [n, k8*8] weight b4 (u32 [n][k8], byte-sliced nibbles) with f32 per-32 scales
 * sw [n][k8/4], times the quantised activation (a8, sa). Bit-exact with
 * engine/reference.py gemv_w4, including numpy's pairwise combine order. */
int hv_a4gv(const int8_t* a8, const float* sa, const uint32_t* b4, const float* sw,
            float* dst, int k8, int n, void* stream);

/* The same GEMV, also writing the exact int32 block dots idot [n][k8/4]
 * (engine/reference.py:66-69). For parity checking. */
int hv_a4gv_idot(const int8_t* a8, const float* sa, const uint32_t* b4, const float* sw,
                 float* dst, int32_t* idot, int k8, int n, void* stream);

/* The engine's weight layout: the same int4 values and scales reordered into 8-row
 * tiles (pair_ffn > 0: 4 gate rows and their 4 up rows of a [gate | up] matrix with
 * 2 * pair_ffn rows), 8 blocks per iteration, so that every warp-wide load of the GEMV
 * reads 512 contiguous bytes. Nothing in the reference corresponds: its GEMV reads the
 * row-major packed form (engine/limited.py:40-58) directly. */
int hv_w4_prepacked_size(int rows, int k, int pair_ffn, size_t* nib_bytes, size_t* scale_bytes);
int hv_w4_prepack(const uint32_t* b4, const float* sw, int rows, int k, int pair_ffn,
                  uint32_t* pb4, float* psw, void* stream);
/* gemv_wpo_a4 over the prepacked layout; dst keeps the reference row order. Matrices of
 * few tiles (under 16 per SM, 4096 <= K <= 16384, K a multiple of 256) run on an
 * iteration-split kernel whose warps share each tile's K; the result is the same bit for
 * bit. */
int hv_a4gv_pp(const int8_t* a8, const float* sa, const uint32_t* pb4, const float* psw,
               float* dst, int k8, int rows, int pair_ffn, void* stream);
/* Prompt prefill: the same GEMV for ntok tokens at once, dst [ntok][rows] (row order as
 * hv_a4gv_pp, [gate | up] for a paired matrix). a8 [ntok][K] int8 and sa [ntok][2 K/32]
 * hold each token's quant_a8s output (scales, then block sums), one row per token. Each
 * token's row is bit-identical to hv_a4gv_pp on that token. K a multiple of 256, at most
 * 32768. The reference has no batched path: it prefills through its decode step one
 * token at a time (engine/limited.py:455-462). */
int hv_a4gemm_pp(const int8_t* a8, const float* sa, const uint32_t* pb4, const float* psw,
                 float* dst, int k8, int rows, int pair_ffn, int ntok, void* stream);
/* The per-token steps of a batched prompt prefill, for ntok tokens (rows) at once. Each
 * applies to every row the arithmetic of the one-token kernel the eager step uses
 * (engine/limited.py:374-419), so a prefill built from them equals the token-by-token
 * prefill bit for bit:
 *   hv_gather_rows  h[t] = f32(emb16[tok[t]])                          (gather_emb)
 *   hv_qa8s_rows    quant_a8s of each row of src [ntok][nb*32]; sa row t = (scales,
 *                   block sums) [2 nb]                                   (quant_a8s)
 *   hv_qk_rows      q/k RMSNorm (eps) + RoPE at position pos0 + t of the qkv rows
 *                   [ntok][(nq + 2 nkv) hd]; q heads to q_out [ntok][nq][hd], k and v
 *                   rows appended at pos0 + t of the f32 cache [nkv][cap][hd]
 *                                                     (rmsnorm_bp, rope_pos, kvapp_pos)
 *   hv_attn_rows    attention of query row t over positions 0 .. pos0 + t, the
 *                   arithmetic of hv_attn_decode at that position; part is caller
 *                   scratch of hv_attn_rows_scratch's part_bytes (ticket is not used
 *                   and may be any pointer)                             (fda_warp_pos)
 *   hv_silu_rows    act[t] = silu(gate[t]) * up[t] from [gate | up] rows (gpu_silu_mul) */
int hv_gather_rows(const uint16_t* emb16, const int32_t* tok, float* h, int hid, int ntok,
                   void* stream);
int hv_qa8s_rows(const float* src, int8_t* a8, float* sa, int nb, int ntok, void* stream);
int hv_qk_rows(const float* qkv, const float* qn, const float* kn, const float* cos_t,
               const float* sin_t, int pos0, float* q_out, float* kc, float* vc, int nq,
               int nkv, int hd, int cap, float eps, int ntok, void* stream);
int hv_attn_rows_scratch(int nq, int group, int cap, int ntok, size_t* part_bytes,
                         size_t* ticket_bytes);
int hv_attn_rows(const float* q, const float* kc, const float* vc, float* ctx,
                 const float* scale, int pos0, int nq, int hd, int group, int kvstride,
                 int ntok, float* part, int32_t* ticket, void* stream);
int hv_silu_rows(const float* gu, float* act, int ffn, int ntok, void* stream);
/* hv_qk_rows and hv_attn_rows over a binary16 cache (the compressed-KV lane; see
 * hv_kv_append_f16): K and V rows are stored rounded to nearest-even binary16, and
 * attention reads the widened values. */
int hv_qk_rows_f16(const float* qkv, const float* qn, const float* kn, const float* cos_t,
                   const float* sin_t, int pos0, float* q_out, uint16_t* kc, uint16_t* vc,
                   int nq, int nkv, int hd, int cap, float eps, int ntok, void* stream);
int hv_attn_rows_f16(const float* q, const uint16_t* kc, const uint16_t* vc, float* ctx,
                     const float* scale, int pos0, int nq, int hd, int group, int kvstride,
                     int ntok, float* part, int32_t* ticket, void* stream);
/* The same GEMV with dp4a block dots instead of tensor-pipe MMAs, over a "dq"
 * arrangement of the same tiles (equal sizes: hv_w4_prepacked_size): in each 8-block
 * iteration, lane 4g + t of the warp finds all four words of blocks 2t and 2t+1 of row g.
 * hv_w4_prepack_dq writes it; hv_a4gv_dq gives results bit-identical to hv_a4gv_pp on
 * the same matrix. No counterpart in the reference (its k_a4gv reads the row-major form). */
int hv_w4_prepack_dq(const uint32_t* b4, const float* sw, int rows, int k, int pair_ffn,
                     uint32_t* pb4, float* psw, void* stream);
/* hv_a4gemm_pp over weights in the dq arrangement (same results). */
int hv_a4gemm_dq(const int8_t* a8, const float* sa, const uint32_t* pb4, const float* psw,
                 float* dst, int k8, int rows, int pair_ffn, int ntok, void* stream);
int hv_a4gv_dq(const int8_t* a8, const float* sa, const uint32_t* pb4, const float* psw,
               float* dst, int k8, int rows, int pair_ffn, void* stream);
/* hv_a4gv_pp's choice of kernel: 1 (default) lets small matrices use the iteration-split
 * kernel, 0 runs every matrix on the one-warp-per-tile kernel. Process-wide. */
int hv_gemv_set_split(int enable);

/* rmsnorm_bp (k_rmsbp.ptx; launch engine/limited.py:361-362): row-wise
 * dst = w * (src / sqrt(mean(src^2) + eps)); rows x cols; in place allowed. The
 * reference kernel hard-wires eps = 1e-5 (engine/reference.py:34). */
int hv_rmsnorm(const float* src, float* dst, const float* w, int rows, int cols, float eps,
               void* stream);

/* rope_pos (k_devgen.ptx; engine/limited.py:394-397): rotate-half RoPE in place on
 * vec [heads][2*half] at the device position *pos, tables cos/sin [cap][half]. */
int hv_rope(float* vec, const float* cos_t, const float* sin_t, const int32_t* pos, int heads,
            int half, void* stream);

/* kvapp_pos (k_devgen.ptx; engine/limited.py:398-400): KC/VC [nkv][cap][hd] <- k, v at
 * the device position *pos. */
int hv_kv_append(const float* k, const float* v, float* kc, float* vc, const int32_t* pos,
                 int nkv, int hd, int cap, void* stream);

/* fda_warp_pos (k_devgen.ptx; engine/limited.py:401-404): causal decode attention of
 * nq query heads over cache positions 0..*pos, kv head = h / group, logits scaled by
 * *scale, in engine/reference.py:104-118's own order of operations, so ctx is bit for bit
 * the reference's: row dots in OpenBLAS's order (HV_STEP_OPT_REF_BLAS_RUNS), numpy's
 * exp, numpy's pairwise sum, one division per weight, and the weighted V rows summed
 * position by position. Two launches (scores per (kv head, chunk), then the context per
 * (kv head, 32-dim slice)); the library keeps a per-device scratch buffer for the scores
 * (allocated on first use; grow it with hv_attn_reserve before a stream capture). hd must
 * be 128, the cache at most 16384 positions. A *pos outside [0, cap) reads no cache row
 * and leaves NaN in ctx. */
int hv_attn_decode(const float* q, const float* kc, const float* vc, float* ctx,
                   const float* scale, const int32_t* pos, int nq, int hd, int group,
                   int kvstride, void* stream);
/* The compressed-KV lane (no counterpart in the reference, which keeps an f32 cache;
 * engine/limited.py:323-325 names the fp32 KV as the engine's sharpest limitation): the
 * cache holds IEEE binary16 values [nkv][cap][hd] (half the bytes). hv_kv_append_f16
 * stores f16(k), f16(v) rounded to nearest-even (numpy's astype(float16)); then
 * hv_attn_decode_f16 computes exactly what hv_attn_decode computes over an f32 cache that
 * holds those f16 values widened (same chunking, same arithmetic). */
int hv_kv_append_f16(const float* k, const float* v, uint16_t* kc, uint16_t* vc,
                     const int32_t* pos, int nkv, int hd, int cap, void* stream);
int hv_attn_decode_f16(const float* q, const uint16_t* kc, const uint16_t* vc, float* ctx,
                       const float* scale, const int32_t* pos, int nq, int hd, int group,
                       int kvstride, void* stream);

/* Makes sure the attention scratch can serve nkv heads at a cache of `cap` positions. */
int hv_attn_reserve(int nkv, int group, int cap);

/* No counterpart in the reference. hv_attn_decode for callers that cannot let the
 * library allocate (a process that gives all of HBM to its own pool, or a loop that
 * cannot take the device-wide synchronisation of cudaMalloc/cudaFree): same arguments
 * and results, but its scratch is a fixed 2 MiB static device array, so it calls no
 * cudaMalloc or cudaFree. Limit: nq x (cap + chunks) x 4 bytes of scores within 2 MiB
 * (chunks = max(ceil(SMs / nkv), ceil(cap / 1024))); larger problems return
 * HV_E_INVALID. The first call on a device does a one-time set-up (the array's symbol
 * address): make it before any stream capture. All calls on a device share the array;
 * calls that overlap on the GPU race. */
int hv_attn_decode_noalloc(const float* q, const float* kc, const float* vc, float* ctx,
                           const float* scale, const int32_t* pos, int nq, int hd, int group,
                           int kvstride, void* stream);

/* gpu_silu_mul (k_silu.ptx; engine/limited.py:412-413): act = g * sigma(g) * up. */
int hv_silu_mul(const float* gate, const float* up, float* act, int n, void* stream);

/* vec_add (k_vadd.ptx; engine/limited.py:407-408): out = a + b. */
int hv_vadd(const float* a, const float* b, float* out, int n, void* stream);

/* gather_emb (k_devgen.ptx; engine/limited.py:384-385): h = f32(emb16[*tok]). */
int hv_gather_emb(const uint16_t* emb16, const int32_t* tok, float* h, int hid, void* stream);

/* argmax_p (k_devgen.ptx; engine/limited.py:423-425): per-part max of logits[n] into
 * pv/pi [parts], ties to the lowest index. */
int hv_argmax_partial(const float* logits, float* pv, int32_t* pi, int n, int parts,
                      void* stream);
/* argmax_f (k_devgen.ptx; engine/limited.py:426-428): final max over the parts; writes
 * *tok, gen[*step] = tok, then ++*step and ++*pos, all on the device. */
int hv_argmax_final(const float* pv, const int32_t* pi, int32_t* tok, int32_t* gen,
                    int32_t* step, int32_t* pos, int parts, void* stream);

/* Vocabulary-sharded greedy argmax: argmax_p/argmax_f (engine/limited.py:421-428) split
 * at shard boundaries, for an LM head whose rows are spread over several GPUs. The
 * result is np.argmax over the whole vocabulary (engine/reference.py:219: first maximal
 * id; -0 equals +0; a NaN wins, the first one).
 * hv_argmax_key folds logits[0..n) of one shard, whose first row is global id `base`,
 * into *key (atomic max of an order-preserving 64-bit key: value, then lower id).
 * *key must be 0 before the shard's first fold; hv_argmax_key_final leaves it 0. */
int hv_argmax_key(const float* logits, int n, int base, uint64_t* key, void* stream);
/* Max over nkeys shard keys (one per shard, e.g. gathered from every rank), then as
 * argmax_f: *tok, gen[*step] = tok, ++*step, ++*pos; every keys[i] is reset to 0. */
int hv_argmax_key_final(uint64_t* keys, int nkeys, int32_t* tok, int32_t* gen,
                        int32_t* step, int32_t* pos, void* stream);

/* The bounded device-side wait that every cross-CTA and cross-rank wait of the fused
 * step is built on (no counterpart in the reference, whose kernels never wait on each
 * other): one thread polls *word until (*word & mask) == want, for at most limit_ns
 * (0 < limit_ns <= 10 s). If the limit passes it sets *status = HV_E_TIMEOUT (unless
 * *status already holds a failure, which also ends the wait early) and the kernel
 * returns; the context stays usable. Asynchronous: read *status after synchronising.
 * Lets the timeout path be exercised on a word that nothing sets, without a hung GPU. */
int hv_wait_probe(const uint32_t* word, uint32_t mask, uint32_t want, long long limit_ns,
                  int32_t* status, void* stream);

/* quantize_w4 (engine/limited.py:40-58) on the device: f32 w [n][k] -> packed u32
 * [n][k/8] and scales f32 [n][k/32], bit-exact with the host rule. */
int hv_quantize_w4(const float* w, uint32_t* packed, float* scale, int n, int k,
                   void* stream);

/* ---- the fused decode step ---------------------------------------------------------
 *
 * One cooperative launch performs the whole of engine/limited.py Engine._step()
 * (:374-419) and, with HV_STEP_HEAD|HV_STEP_ARGMAX, the LM head and
 * _argmax_into_next() (:421-428): every layer's RMSNorm, quantisation, GEMVs, q/k norm,
 * RoPE, KV append, attention, SiLU and residual adds, then greedy argmax that advances
 * tok/pos/step on the device. One CTA per SM: a producer warp streams the CTA's weight
 * tiles and KV rows into a shared-memory ring with bulk copies while eight consumer
 * warps compute; phases are separated by grid barriers. Every wait (barrier or ring
 * slot) is bounded (HV_E_TIMEOUT, with *status set, instead of a hang). A
 * launch whose *pos is outside [0, cap) or *tok outside [0, vocab) does nothing but set
 * *status = HV_E_INVALID. The host reads *status after synchronising; after a nonzero
 * status, zero `barrier`, `ticket` and `status` before the next launch.
 *
 * Every pointer in these structs is a device pointer; the caller owns all buffers. The
 * hv_step_desc itself is a host struct passed by value into the launch (capturable in a
 * CUDA graph); its `layers` table lives in device memory. */

typedef struct hv_layer_w {
  const uint32_t* qkv_b4; const float* qkv_sw;   /* rows [q | k | v], K = hidden   */
  const uint32_t* o_b4;   const float* o_sw;     /* hidden rows, K = n_head*hd     */
  const uint32_t* gu_b4;  const float* gu_sw;    /* rows [gate | up], K = hidden   */
  const uint32_t* dn_b4;  const float* dn_sw;    /* hidden rows, K = ffn           */
  const float* an; const float* fn;              /* input / post-attention norms   */
  const float* qn; const float* kn;              /* per-head q / k norms [hd]      */
  float* kc; float* vc;                          /* KV cache [n_kv][cap][hd]: f32, or
                                                    binary16 when the step's kv_dtype
                                                    is HV_KV_F16                     */
} hv_layer_w;

typedef struct hv_step_desc {
  int n_layer, hidden, ffn, n_head, n_kv, head_dim, head_rows, cap;
  float eps, attn_scale;
  int attn_chunks;              /* chunks per kv head (hv_step_config)            */
  int vocab;                    /* embedding rows: *tok must lie in [0, vocab)     */
  const hv_layer_w* layers;     /* [n_layer]                                       */
  const uint16_t* emb16;        /* [vocab][hidden] f16                             */
  const float* onorm;           /* final norm [hidden]                             */
  const uint32_t* head_b4; const float* head_sw;   /* LM head [head_rows][hidden] */
  const float* cos_t; const float* sin_t;          /* RoPE tables [cap][hd/2]      */
  int32_t* tok; int32_t* pos; int32_t* step;      /* device scalars                  */
  int32_t* gen;                 /* generated tokens [cap + 1]                      */
  float* h;                     /* residual [hidden]                               */
  float* qkv;                   /* [(n_head + 2 n_kv) hd]                          */
  float* ctx;                   /* room for [n_head hd] floats (whole, all ranks); the
                                   step keeps the attention output there quantised:
                                   int8 [n_head hd] then (scale, sum) per 32 values  */
  float* act;                   /* room for [ffn] floats (whole); holds the SiLU output
                                   quantised the same way                           */
  float* logits;                /* [head_rows]                                     */
  float* part;                  /* attention scratch (hv_step_config): scores
                                   [n_head][cap], then chunk maxima [n_head][chunks] */
  int32_t* ticket;              /* [2 n_kv + 1] zeroed once; every launch leaves them
                                   zero (after a failed launch the caller re-zeroes) */
  float* amax_v; int32_t* amax_i;                  /* [grid] argmax partials       */
  uint32_t* barrier;            /* four words, zeroed once                         */
  int32_t* status;              /* 0 = ok; nonzero after a bounded wait ran out    */
  uint64_t* trace;              /* NULL, or [grid][HV_STEP_TRACE_STRIDE(n_layer)]:
                                   %globaltimer (ns) at each phase boundary, per CTA */
  const void* plans;            /* hv_step_plans() output, uploaded to the device  */
  /* Column-parallel sharding over `world` GPUs (world 1 = one GPU, `peers` unused).
   * Rank r holds q heads [r nq, (r+1) nq) and kv heads [r nkv, (r+1) nkv) with nq =
   * n_head and nkv = n_kv (per-rank counts), rows [r hidden/world, ...) of W_o and
   * W_down, gate/up rows [r ffn, (r+1) ffn) with ffn per rank, and LM-head rows
   * [r head_rows, ...); every output element is still computed whole on one GPU. The
   * step writes each produced slice into every rank's copy (NVLink peer stores) and its
   * grid barrier spans all ranks' CTAs, so the all-gathers are part of the kernel. */
  int world, rank;
  const struct hv_step_peers* peers;   /* device pointer (world > 1) */
  /* Element type of every layer's kc/vc: HV_KV_F32 (0, the reference's cache) or
   * HV_KV_F16 (the compressed-KV lane: this step's k and v rows are rounded to binary16,
   * appended as such, and attention reads every row as the widened binary16 value --
   * the arithmetic of hv_kv_append_f16 followed by hv_attn_decode_f16). */
  int kv_dtype;
  /* Arrangement of every prepacked weight tile: HV_W4_PP (0, hv_w4_prepack, block dots
   * on the tensor pipe) or HV_W4_DQ (hv_w4_prepack_dq, dp4a block dots; same results). */
  int w4_layout;
  /* The KV cache seen as one array of rows of head_dim elements (of kv_dtype): every
   * layer's kc and vc lie within kv_rows rows from kv_base (16-byte aligned). The step
   * copies 32-dim slices of V rows out of it with the tensor-copy engine. */
  const void* kv_base;
  long long kv_rows;
} hv_step_desc;

#define HV_KV_F32 0
#define HV_KV_F16 1
#define HV_W4_PP 0
#define HV_W4_DQ 1

#define HV_MAX_WORLD 8
/* Every rank's copies of the exchanged buffers (device pointers valid on this rank:
 * its own allocations and the other ranks' opened with hv_ipc_open). */
typedef struct hv_step_peers {
  float* h[HV_MAX_WORLD];          /* residual [hidden]                              */
  void* ctx[HV_MAX_WORLD];         /* quantised attention output (desc.ctx buffers)  */
  void* act[HV_MAX_WORLD];         /* quantised SiLU output (desc.act buffers)       */
  uint32_t* barrier[HV_MAX_WORLD]; /* every rank's desc.barrier (four words)         */
  int32_t* xchg[HV_MAX_WORLD];     /* argmax exchange [HV_MAX_WORLD + 1][4], zeroed once */
} hv_step_peers;

/* Trace layout: entry 0 = kernel start, 1 = set-up done; layer l at 2 + 28 l:
 * +0 qkv prologue, +1 qkv GEMV, +2 barrier, +3 attention, +4 barrier, +5 o prologue,
 * +6 o GEMV, +7 barrier, +8 gate/up prologue, +9 gate/up GEMV, +10 barrier,
 * +11 down prologue, +12 down GEMV, +13 barrier; inside the attention (last work item
 * of the CTA): +14 q/k norms and RoPE, +15 scores, +16 scores stored and ticket taken;
 * on the CTAs of a context item: +17 its kv head's scores all in, +18 exps and pairwise
 * leaves done, +19 weighted V chain and quantisation done (all %globaltimer ns).
 * Durations (ns) that consumer warp 0 spent waiting for its shared-memory ring slots:
 * +21 attention scores, +23 qkv GEMV, +24 gate/up GEMV (+20 is scratch); +25 = SM
 * cycles warp 0 spent computing attention scores; +26 / +27: inside the qkv prologue,
 * vector loaded and squared / sum of squares done. Then
 * the head prologue, head GEMV and argmax at 2 + 28 n_layer + {0, 1, 2}; then, for the
 * producer warp: ns blocked on a ring slot still in use (+3), ns blocked on the copies in
 * flight (+4), slots copied (+5); for a context item's CTA, over the whole launch: ns its
 * warp 0 waited for V slots (+6), ns of its exps and leaf sums (+7). */
#define HV_STEP_TRACE_STRIDE(n_layer) (10 + 28 * (n_layer))

#define HV_STEP_HEAD 1     /* compute the LM head into logits                          */
#define HV_STEP_ARGMAX 2   /* then greedy argmax: tok = argmax, gen[step] = tok,
                              ++step, ++pos (engine/limited.py:421-428)               */

/* Launch geometry of the fused step on the current device, and the sizes of the
 * scratch it needs: `part_floats` floats for hv_step_desc.part, `chunks` for
 * attn_chunks, `grid` entries for amax_v / amax_i. */
int hv_step_config(int n_kv, int group, int cap, int* grid, int* threads, size_t* smem,
                   int* chunks, size_t* part_floats);

/* The step's reduction plans (numpy's pairwise order for RMSNorm over `hidden` and for
 * GEMV rows of K = hidden, qdim, ffn) into a host buffer of hv_step_plans_bytes() bytes;
 * the caller uploads it and points hv_step_desc.plans at the device copy. */
int hv_step_plans_bytes(size_t* bytes);
int hv_step_plans(int hidden, int qdim, int ffn, void* host_buf, size_t len);

/* One fused decode step. `desc` is a host pointer to a filled hv_step_desc. */
int hv_step_launch(const hv_step_desc* desc, int flags, void* stream);

/* Tuning of later hv_step_launch calls (process-wide): HV_STEP_OPT_INFLIGHT = bulk copies
 * each CTA's producer keeps in flight (1..32, default 6); HV_STEP_OPT_EVICT_FIRST = mark
 * the streamed weights and KV rows evict-first in L2 (0/1, default 1);
 * HV_STEP_OPT_LOCAL_QKV_BARRIER = in a sharded step, meet only the rank's own CTAs after
 * the qkv projection (attention reads no other rank's data; 0/1, default 0). None changes
 * any result. No counterpart in the reference (its kernels have no such knobs). */
#define HV_STEP_OPT_INFLIGHT 1
#define HV_STEP_OPT_EVICT_FIRST 2
#define HV_STEP_OPT_LOCAL_QKV_BARRIER 3
/* HV_STEP_OPT_REF_BLAS_RUNS: the OpenBLAS thread count of the host whose reference results
 * the attention reproduces bit for bit (default 8). The reference's `keys @ q` splits a
 * gemv of T rows into that many runs when 128 T >= 460800, and the row dot of each run's
 * last rows takes another order; every attention entry point (decode, rows, no-alloc and
 * the fused step) follows the same setting. Process-wide. */
#define HV_STEP_OPT_REF_BLAS_RUNS 5
int hv_step_set_option(int option, int value);

#ifdef __cplusplus
}
#endif

#endif /* HIVE_B200_H */
