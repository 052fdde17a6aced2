/*
 * pu_attn.h — C ABI of the B200 (sm_100a) attention library `libpu_attn.so`.
 *
 * This is the drop-in boundary for the attention hot path of Pallas-Unbound
 * (a JAX/Pallas TPU project).  The reference exposes two jitted Python
 * functions and no native ABI; each entry point below names the reference
 * function (file:line inside the reference project) whose work it replaces.
 * A JAX FFI handler, a ctypes stub or a torch op binds these symbols; the
 * Python package `pallas_flash` in this repository is the ctypes binding.
 *
 * Conventions shared by every entry point
 *   - Every tensor is a plain device pointer to a dense row-major array.
 *     Attention tensors use the reference layout [B, H, N, D]
 *     (src/pallas_flash/ops/interface.py:27, kernels/decoding.py:111).
 *   - The caller owns every buffer.  No entry point allocates device memory
 *     (except pu_peer_alloc, whose purpose is an IPC-exportable buffer) or
 *     synchronises the host; all work is enqueued on `stream`
 *     (a cudaStream_t, NULL = legacy default stream).
 *   - Return value: PU_OK (0) or a PU_ERR_* code; pu_last_error() gives a
 *     human-readable message for the calling thread.
 *   - Device-side waits are bounded.  A wait that runs out records
 *     PU_ERR_DEVICE_TIMEOUT in a per-device status word that
 *     pu_device_status() reads and clears.
 *   - Thread-safe across devices; one stream per call.
 */
#ifndef PU_ATTN_H_
#define PU_ATTN_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define PU_API __attribute__((visibility("default")))
#else
#define PU_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define PU_OK 0
#define PU_ERR_INVALID_ARGUMENT 1
#define PU_ERR_UNSUPPORTED 2
#define PU_ERR_CUDA 3
#define PU_ERR_WORKSPACE 4
#define PU_ERR_DEVICE_TIMEOUT 5

/* element types */
#define PU_DTYPE_BF16 0
#define PU_DTYPE_F16 1
#define PU_DTYPE_F32 2
#define PU_DTYPE_FP8_E4M3 3   /* KV caches of pu_decode_gqa only */

/* Number of floats in one packed split-KV partial record: m, l, o[D]. */
#define PU_PARTIAL_FLOATS(D) ((D) + 2)

/*
 * Library identity: returns a static string with the build's target
 * architecture and version.  No reference counterpart.
 */
PU_API const char* pu_version(void);

/*
 * Architecture of the machine code the current device would run for this
 * library's kernels (cudaFuncGetAttributes binaryVersion of every kernel,
 * major*10 + minor; 100 for sm_100a), written to *arch.  Returns an error if
 * the kernels disagree or cannot be loaded.  No reference counterpart.
 */
PU_API int pu_binary_arch(int* arch);

/* Message for the last error raised on the calling thread ("" if none). */
PU_API const char* pu_last_error(void);

/*
 * Synchronises the current device, then returns (and clears) its device
 * status word: PU_OK, or PU_ERR_DEVICE_TIMEOUT when a kernel gave up on a
 * bounded wait.  `*detail` (optional) receives the kernel's location code.
 * No reference counterpart (the reference surfaces errors as XLA exceptions,
 * tests/test_memory.py:59-69).
 */
PU_API int pu_device_status(int* detail);

/*
 * Failure-detection self-test (no reference counterpart): launches one CTA
 * that waits, with the same bounded mbarrier wait the attention kernels
 * use, on a barrier nothing completes, giving up after `timeout_ns`
 * (<= 2 s).  A following pu_device_status() returns PU_ERR_DEVICE_TIMEOUT
 * with detail 901; the CUDA context remains usable.
 */
PU_API int pu_selftest_wait_timeout(uint64_t timeout_ns, void* stream);

/*
 * Training attention forward.
 * Replaces pallas_flash_attention (src/pallas_flash/ops/interface.py:20-85),
 * whose kernel is flash_attention_kernel (kernels/attention.py:11-36) running
 * the online-softmax loop pipeline_kv_loop (kernels/pipeline.py:14-60).
 *   q [B,H,Nq,D], k/v [B,H,Nkv,D], o [B,H,Nq,D]: bf16.
 *   lse [B,H,Nq] fp32 natural-log LogSumExp of the scaled logits, or NULL.
 *   D must be 64 or 128 (the host pads other head sizes, as the reference's
 *   layout.pad_tensor does).  Any Nq, Nkv >= 1.
 *   sm_scale multiplies q.k (the reference folds 1/sqrt(D) into q,
 *   interface.py:43-44).  causal != 0 masks key j > query i (the causal
 *   semantics of benchmarks/baseline_mha.py:47-50, top-left aligned).
 */
PU_API int pu_attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
                int64_t B, int64_t H, int64_t Nq, int64_t Nkv, int64_t D,
                float sm_scale, int causal, void* stream);

/*
 * Bytes of device workspace pu_attn_bwd (and pu_attn_bwd_deterministic)
 * needs: the row statistics LSE*log2(e) and Delta = rowsum(dO*O), and for
 * D = 128 an fp32 dQ accumulator [B*H][Nq rounded up to 128][D].
 */
PU_API size_t pu_attn_bwd_workspace_size(int64_t B, int64_t H, int64_t Nq, int64_t D);

/*
 * Training attention backward: dQ, dK, dV (bf16) from q, k, v, o, lse and dO.
 * The reference has no backward kernel (forward only, no custom_vjp); this
 * replaces the autodiff of benchmarks/baseline_mha.py:22-58.
 *   workspace: >= pu_attn_bwd_workspace_size() bytes, 256-byte aligned;
 *   its contents need not be initialised.
 * For D = 128 one fused pass computes all five products of every (key
 * tile, query tile) pair and adds dQ into the fp32 accumulator with
 * reductions in L2, so dQ's last bits depend on the order in which key
 * tiles finish (dK and dV are deterministic); D = 64 runs the two-kernel
 * path of pu_attn_bwd_deterministic.
 */
PU_API int pu_attn_bwd(const void* q, const void* k, const void* v, const void* o,
                const float* lse, const void* dout,
                void* dq, void* dk, void* dv,
                void* workspace, size_t workspace_bytes,
                int64_t B, int64_t H, int64_t Nq, int64_t Nkv, int64_t D,
                float sm_scale, int causal, void* stream);

/*
 * The same gradients, bitwise reproducible run to run (same replacement of
 * the autodiff of benchmarks/baseline_mha.py:22-58): a dK/dV kernel per key
 * tile and a dQ kernel per query tile, each gradient element written once
 * with no atomics.  S and dP are computed in both kernels, so it performs 7
 * of the 128x128xD products per tile pair instead of 5 and is slower.
 * Same arguments and workspace as pu_attn_bwd.
 */
PU_API int pu_attn_bwd_deterministic(const void* q, const void* k, const void* v, const void* o,
                const float* lse, const void* dout,
                void* dq, void* dk, void* dv,
                void* workspace, size_t workspace_bytes,
                int64_t B, int64_t H, int64_t Nq, int64_t Nkv, int64_t D,
                float sm_scale, int causal, void* stream);

/*
 * Bytes of device workspace the split-KV decode entry points need for a
 * cache shard of n_local tokens.
 */
PU_API size_t pu_decode_workspace_size(int64_t B, int64_t H, int64_t n_local, int64_t D);

/*
 * Split-KV decode partial for one shard of the KV cache.
 * Replaces decoding_kv_loop (src/pallas_flash/kernels/decoding.py:19-60),
 * which returns (o, m, l) per (b, h); the reference discards m, l
 * (decoding.py:73) — here they are the shard's output.
 *   q [B,H,1,D] (q_dtype), k_cache/v_cache [B,H,n_local,D] (kv_dtype):
 *   PU_DTYPE_F16 or PU_DTYPE_BF16.  D must be 128 or 64.
 *   kv_lens: int32[B] device array of global sequence lengths, or NULL
 *   (every sequence is kv_offset + n_local long).  Token t of this shard
 *   has global position kv_offset + t and is masked when >= kv_lens[b]
 *   (the padding mask of decoding.py:42-44).
 *   partial: fp32 [B*H][D+2] records {m, l, o[D]}: m = max scaled logit
 *   (natural-log units), l = sum exp(s - m), o = sum exp(s - m) v
 *   (unnormalised).  An empty shard gives m = -inf, l = 0, o = 0.
 *   workspace: >= pu_decode_workspace_size() bytes; it must be zero-filled
 *   before its first use and is left zero-filled by every call that returns
 *   PU_OK and completes on the device.
 */
PU_API int pu_decode_partial(const void* q, int q_dtype,
                      const void* k_cache, const void* v_cache, int kv_dtype,
                      const int32_t* kv_lens, int64_t kv_offset,
                      float* partial, void* workspace, size_t workspace_bytes,
                      int64_t B, int64_t H, int64_t n_local, int64_t D,
                      float sm_scale, void* stream);

/*
 * Stable LogSumExp merge of G gathered shard partials into the attention
 * output.  Replaces the documented-only psum merge of the reference
 * (README.md:41-46, docs/project_plan.md:219-225); the algebra is the
 * online-softmax update of kernels/pipeline.py:47-52 applied across shards.
 *   partials: fp32 [G][B*H][D+2] (the layout an all-gather of
 *   pu_decode_partial outputs produces).
 *   o: bf16 [B,H,1,D] (the reference's output dtype, decoding.py:83-84).
 *   lse: fp32 [B,H] natural-log LogSumExp, or NULL.
 */
PU_API int pu_decode_combine(const float* partials, int64_t G, void* o, float* lse,
                      int64_t B, int64_t H, int64_t D, void* stream);

/*
 * Library-owned NCCL communicator for the gather between pu_decode_partial
 * and pu_decode_combine, for callers with no communicator of their own.
 * Replaces the cross-device exchange of the reference's sharded decode: its
 * psum/all_gather wrappers (src/pallas_flash/distributed/collectives.py:27-117)
 * and the documented split-KV merge (README.md:41-46).  NCCL is loaded at
 * first use (libnccl.so.2, the process's copy if one is loaded); without it
 * these return PU_ERR_UNSUPPORTED.
 *   pu_comm_unique_id: one rank creates the id (PU_COMM_ID_BYTES bytes) and
 *     shares it with the others over any host channel.
 *   pu_comm_init: every rank, with its own device current, joins; blocks
 *     until all nranks ranks have joined.
 *   pu_allgather_partials: partial fp32 [B*H][D+2] of this rank ->
 *     gathered fp32 [nranks][B*H][D+2] on every rank (rank order), on stream.
 *   pu_comm_destroy: after the last use on every rank.
 */
#define PU_COMM_ID_BYTES 128
PU_API int pu_comm_unique_id(void* id);
PU_API int pu_comm_init(const void* id, int64_t nranks, int64_t rank, void** comm);
PU_API int pu_allgather_partials(const float* partial, float* gathered, int64_t B, int64_t H,
                                 int64_t D, void* comm, void* stream);
PU_API int pu_comm_destroy(void* comm);

/*
 * Single-GPU decode step: pu_decode_partial over the whole cache with the
 * merge fused into the same kernel (the last CTA of each (b, h) combines).
 * Replaces pallas_flash_decoding (src/pallas_flash/kernels/decoding.py:105-145).
 *   o bf16 [B,H,1,D]; lse fp32 [B,H] or NULL; workspace as above.
 */
PU_API int pu_decode(const void* q, int q_dtype,
              const void* k_cache, const void* v_cache, int kv_dtype,
              const int32_t* kv_lens, void* o, float* lse,
              void* workspace, size_t workspace_bytes,
              int64_t B, int64_t H, int64_t n, int64_t D,
              float sm_scale, void* stream);

/*
 * Single-GPU decode step with grouped K/V heads and optional fp8 caches.
 * No counterpart in the reference (its decode has one K/V head per query
 * head and a bf16 cache, kernels/decoding.py:105-115); same step as
 * pu_decode otherwise.
 *   q [B,H,1,D] f16/bf16; k_cache/v_cache [B,H_kv,n,D] with H % H_kv == 0:
 *   query head h reads K/V head h / (H / H_kv) (GQA; H_kv = 1 is MQA).
 *   kv_dtype: PU_DTYPE_F16, PU_DTYPE_BF16 or PU_DTYPE_FP8_E4M3; the stored
 *   values times k_scale / v_scale are the keys / values (per-tensor
 *   scales; pass 1 for f16/bf16).
 *   With H / H_kv = 2, 4 or 8 one CTA serves all query heads of a K/V head,
 *   so each K/V byte is read from DRAM once.
 *   o bf16 [B,H,1,D]; lse fp32 [B,H] or NULL; workspace of
 *   pu_decode_gqa_workspace_size(B, H, H_kv, n, D) bytes, zeroed before its
 *   first use (left zeroed, as for pu_decode).
 */
/* Bytes of workspace pu_decode_gqa needs (0 on invalid sizes). */
PU_API size_t pu_decode_gqa_workspace_size(int64_t B, int64_t H, int64_t H_kv, int64_t n, int64_t D);

PU_API int pu_decode_gqa(const void* q, int q_dtype,
                         const void* k_cache, const void* v_cache, int kv_dtype,
                         const int32_t* kv_lens, void* o, float* lse,
                         void* workspace, size_t workspace_bytes,
                         int64_t B, int64_t H, int64_t H_kv, int64_t n, int64_t D,
                         float sm_scale, float k_scale, float v_scale, void* stream);

/*
 * Allocation-free single-GPU decode step.  No counterpart in the reference:
 * it exists for callers that have no way to hand over device scratch memory
 * — for example a custom-call handler that receives only its operand and
 * result buffers, or a serving runtime that plans all device memory at
 * start-up and forbids allocation afterwards.  Same inputs, outputs and
 * results as pu_decode, without the workspace arguments.
 *   Scratch: a fixed 8 MiB array in the library's device memory, present on
 *   every GPU that loads the library until the process exits.  A call needs
 *   256 KiB + B*H*splits*(D+2)*4 bytes (splits = the split count pu_decode
 *   chooses on a 148-SM B200: floor(296 / (B*H)) without kv_lens, about
 *   ceil(1184 / (B*H)) with kv_lens, at least 1); larger problems are
 *   rejected with PU_ERR_WORKSPACE and a message, before anything is enqueued.
 *   The entry point allocates nothing (no cudaMalloc/cudaFree, no library
 *   allocator); it clears the scratch counters with cudaMemsetAsync on
 *   `stream` before the kernel.
 *   Set-up: the first call on each device looks up the array's device
 *   address (cudaGetSymbolAddress) with that device current; make that first
 *   call before any stream capture begins.
 *   All calls on a device share the one array, so calls that overlap on the
 *   GPU (different streams, no ordering between them) race and must not be
 *   issued.
 */
PU_API int pu_decode_noalloc(const void* q, int q_dtype,
                             const void* k_cache, const void* v_cache, int kv_dtype,
                             const int32_t* kv_lens, void* o, float* lse,
                             int64_t B, int64_t H, int64_t n, int64_t D,
                             float sm_scale, void* stream);

/*
 * Paged KV cache.  No counterpart in the reference: its decode reads a
 * dense, padded [B,H,N,D] cache (src/pallas_flash/kernels/decoding.py:86-103,
 * 113-115) and has no cache-update op.  A paged cache lets sequences grow
 * without copying the cache:
 *   k_pool, v_pool: [num_pages][H][page_size][D], fp16 or bf16 (kv_dtype);
 *     page p, head h holds page_size consecutive tokens of one sequence.
 *   page_table: int32 [B][max_pages_per_seq]; entry i of sequence b is the
 *     physical page of tokens [i*page_size, (i+1)*page_size).
 *   kv_lens: int32 [B], tokens held by each sequence (required).
 *   page_size: a power of two in [16, 4096].
 * Only the first ceil(kv_lens[b] / page_size) table entries of a sequence
 * are read.  An entry outside [0, num_pages) is not followed: the kernel
 * records PU_ERR_INVALID_ARGUMENT in the device status word
 * (pu_device_status, detail 302 for decode, 303 for append) and skips those
 * tokens.
 */

/* Bytes of workspace pu_decode_paged needs (0 on invalid sizes). */
PU_API size_t pu_decode_paged_workspace_size(int64_t B, int64_t H, int64_t max_pages_per_seq,
                                             int64_t page_size, int64_t D);

/*
 * Decode step over a paged cache: same results as pu_decode on the dense
 * cache the pages describe.  q [B,H,1,D] f16/bf16; o bf16 [B,H,1,D];
 * lse fp32 [B,H] or NULL; workspace zeroed before its first use (the
 * kernel leaves it zeroed).
 */
PU_API int pu_decode_paged(const void* q, int q_dtype,
                           const void* k_pool, const void* v_pool, int kv_dtype,
                           const int32_t* page_table, int64_t max_pages_per_seq,
                           int64_t num_pages, int64_t page_size,
                           const int32_t* kv_lens, void* o, float* lse,
                           void* workspace, size_t workspace_bytes,
                           int64_t B, int64_t H, int64_t D,
                           float sm_scale, void* stream);

/*
 * Append one token per sequence to a paged cache: writes k_new/v_new
 * [B,H,1,D] (kv_dtype) at position kv_lens[b] (page
 * page_table[b][kv_lens[b] / page_size]) of every head, then advances
 * kv_lens[b] by one, all on `stream`.  The caller maps a page into the
 * table before a sequence crosses into it; a position past the table
 * (kv_lens[b] >= max_pages_per_seq * page_size) or an invalid entry is
 * reported as above and leaves that sequence unchanged.
 */
PU_API int pu_kv_append(const void* k_new, const void* v_new, int kv_dtype,
                        void* k_pool, void* v_pool,
                        const int32_t* page_table, int64_t max_pages_per_seq,
                        int64_t num_pages, int64_t page_size, int32_t* kv_lens,
                        int64_t B, int64_t H, int64_t D, void* stream);

/*
 * Sequence-sharded decode over NVLink peer memory (replaces the all-gather
 * between pu_decode_partial and pu_decode_combine).  Replaces the same
 * reference step as those two: the split-KV LogSumExp merge documented in
 * README.md:41-46 for the mesh-sharded decode (kernels/decoding.py:105-145
 * under distributed/mesh.py:57-77), which the reference never implements.
 *
 * Each of the G ranks (one process per GPU, G <= 8, GPUs with peer access)
 * owns one exchange buffer of pu_decode_exchange_bytes(B,H,D,G) bytes,
 * allocated zeroed by pu_peer_alloc, whose IPC handle it shares with the
 * other ranks (any host channel); each rank opens the others' handles with
 * pu_peer_open.  Per decode step, every rank calls, on its own stream and
 * with the same epoch (1, 2, 3, ... in lockstep):
 *   pu_decode_push: the split-KV pass over the local shard; the record of
 *     each (b, h) is stored into every rank's exchange buffer as 64-bit
 *     words {value, epoch}.  exchange[g] = this process's pointer to rank
 *     g's buffer (its own allocation for g == rank).
 *   pu_decode_pull: waits until all G ranks have published this epoch
 *     (bounded by timeout_ns <= 2 s; on expiry pu_device_status reports
 *     PU_ERR_DEVICE_TIMEOUT, detail 304, and o is zeros), then merges the
 *     records exactly as pu_decode_combine: same o / lse on every rank.
 * A rank must not free or close buffers while another rank may still push.
 */
#define PU_IPC_HANDLE_BYTES 64

/* cudaMalloc + zero-fill a buffer and export its IPC handle (64 bytes). */
PU_API int pu_peer_alloc(size_t bytes, void** dev_ptr, void* ipc_handle);
PU_API int pu_peer_free(void* dev_ptr);
/* Map another process's buffer (peer access enabled on first use). */
PU_API int pu_peer_open(const void* ipc_handle, void** dev_ptr);
PU_API int pu_peer_close(void* dev_ptr);

PU_API size_t pu_decode_exchange_bytes(int64_t B, int64_t H, int64_t D, int64_t G);

PU_API int pu_decode_push(const void* q, int q_dtype,
                          const void* k_cache, const void* v_cache, int kv_dtype,
                          const int32_t* kv_lens, int64_t kv_offset,
                          void* const* exchange, int64_t G, int64_t rank, uint32_t epoch,
                          void* workspace, size_t workspace_bytes,
                          int64_t B, int64_t H, int64_t n_local, int64_t D,
                          float sm_scale, void* stream);

PU_API int pu_decode_pull(const void* exchange, int64_t G, uint32_t epoch,
                          void* o, float* lse, int64_t B, int64_t H, int64_t D,
                          uint64_t timeout_ns, void* stream);

/*
 * One sharded decode step: pu_decode_push followed by the merge.  When B*H
 * is at most half of the GPU's resident split-KV CTAs (148 on a B200) the
 * merge runs inside the push kernel (the last CTA of each (b, h) waits for
 * the other ranks' records), otherwise as pu_decode_pull.  Same results.
 */
PU_API int pu_decode_sharded(const void* q, int q_dtype,
                             const void* k_cache, const void* v_cache, int kv_dtype,
                             const int32_t* kv_lens, int64_t kv_offset,
                             void* const* exchange, int64_t G, int64_t rank, uint32_t epoch,
                             void* o, float* lse, void* workspace, size_t workspace_bytes,
                             int64_t B, int64_t H, int64_t n_local, int64_t D,
                             float sm_scale, uint64_t timeout_ns, void* stream);

/*
 * Attention output projection fused with the tensor-parallel all-reduce.
 * Replaces the partial out-projection + all_reduce_tp (psum over the 'tp'
 * axis) of src/pallas_flash/distributed/collectives.py:27-41, the step after
 * attention when heads are sharded over devices.
 *
 * G ranks (one process per GPU, G <= 8, peer access between the GPUs) each
 * hold o_local [T, K] (this rank's heads' attention output) and w_local
 * [K, N] (the matching rows of W_O), bf16 row-major; every rank receives
 * y = sum_g o_g w_g [T, N] bf16 (identical on all ranks).  T must be a
 * multiple of 128, N of 256, K of 64.  The exchange buffers are set up as
 * for pu_decode_push (pu_peer_alloc / pu_peer_open) with
 * pu_outproj_exchange_bytes(T, N, G) bytes each; exchange[g] = this
 * process's pointer to rank g's buffer.  All ranks call with the same epoch
 * (1, 2, 3, ... in lockstep).  One tcgen05 GEMM kernel stores each bf16
 * partial tile into its owner's buffer over NVLink, the owners reduce and
 * broadcast, and every rank copies the result into y; each wait is bounded
 * by timeout_ns (<= 2 s): on expiry pu_device_status reports
 * PU_ERR_DEVICE_TIMEOUT, detail 401.  For T a multiple of 256 the GEMM runs
 * on CTA pairs (clusters of two SMs, 256 x 256 tiles); the environment
 * variable PU_OUTPROJ_PAIR=0 selects the single-CTA kernel for every T.
 */
PU_API size_t pu_outproj_exchange_bytes(int64_t T, int64_t N, int64_t G);

PU_API int pu_outproj_allreduce(const void* o_local, const void* w_local, void* y,
                                void* const* exchange, int64_t G, int64_t rank, uint32_t epoch,
                                int64_t T, int64_t K, int64_t N, uint64_t timeout_ns,
                                void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PU_ATTN_H_ */
