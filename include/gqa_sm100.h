/*
 * gqa_sm100.h -- C ABI of libgqa_sm100.so, the B200 (sm_100a) GQA
 * flash-attention forward.
 *
 * Conventions shared by every entry point:
 *   - All pointers are device pointers owned by the caller; the library never
 *     allocates device memory. Kernels that need scratch take a caller-owned
 *     workspace (see *_workspace_bytes).
 *   - Tensors use the reference layout: Q/O (batch, num_heads, seq_q, head_dim),
 *     K/V (batch, num_kv_heads, seq_kv, head_dim). Strides are in ELEMENTS, in
 *     dimension order (b, h, s, d). The d stride must be 1 and every other
 *     stride a multiple of 8 elements (16 bytes); base pointers 16-byte aligned.
 *   - dtype: GQA_DTYPE_F16 or GQA_DTYPE_BF16 (q, k, v and o share it).
 *   - scale_log2 = head_dim^-0.5 * log2(e); the softmax is evaluated with exp2.
 *   - causal = 1: query row i (in key coordinates i + seq_kv - seq_q) attends
 *     to keys [0, i + seq_kv - seq_q] (bottom-right alignment). A row with no
 *     visible key produces NaN, as the reference does.
 *   - Work is enqueued on `stream` (a cudaStream_t; NULL = legacy default);
 *     no entry point synchronises. Return 0 on success or a GQA_ERR_* code;
 *     gqa_strerror() turns a code into text.
 *   - Entry points are stateless and re-entrant; per-device attributes are
 *     cached once under a mutex.
 */
#ifndef GQA_SM100_H_
#define GQA_SM100_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GQA_OK 0
#define GQA_ERR_INVALID_ARG 1   /* bad shape, null pointer, negative size      */
#define GQA_ERR_UNSUPPORTED 2   /* head_dim not 64/128, group size not 2^k ... */
#define GQA_ERR_ALIGNMENT 3     /* stride or base pointer not 16-byte aligned  */
#define GQA_ERR_CUDA 4          /* a CUDA runtime/driver call failed           */
#define GQA_ERR_TIMEOUT 5       /* a bounded in-kernel wait expired            */
#define GQA_ERR_WORKSPACE 6     /* workspace missing or too small              */
#define GQA_ERR_NO_DEVICE 7     /* no sm_100 device current                    */
#define GQA_ERR_SCRATCH_LIMIT 8 /* problem needs more than the static scratch  */
#define GQA_ERR_DEBUG_CHECK 9   /* a debug build's address/coordinate check failed (device error word) */

#define GQA_DTYPE_F16 0
#define GQA_DTYPE_BF16 1

/* Text for a status code (static storage). */
const char* gqa_strerror(int code);

/* Library version, major*10000 + minor*100 + patch (0.1.0 -> 100). */
int gqa_version(void);

/*
 * Single-pass GQA forward: O = softmax(Q K^T * scale) V with the group's
 * query heads packed into the M dimension of each tile.
 * Replaces the launch of gqa_fwd_kernel in gqa_kernels/dispatch.py:50-61
 * (kernel body gqa_kernels/gqa_fwd.py:33-109).
 * Packed rows (group_size * seq_q) >= 128 run the tcgen05/TMEM prefill
 * kernel; fewer run the HBM-streaming kernel, which may split the key range
 * across CTAs when `workspace` is large enough
 * (gqa_fwd_workspace_bytes) -- the combine is fused into the same launch.
 */
size_t gqa_fwd_workspace_bytes(int batch, int num_heads, int num_kv_heads, int seq_q, int seq_kv,
                               int head_dim);
int gqa_fwd(const void* q, const void* k, const void* v, void* o, const int64_t* q_strides4,
            const int64_t* k_strides4, const int64_t* v_strides4, const int64_t* o_strides4, int batch,
            int num_heads, int num_kv_heads, int seq_q, int seq_kv, int head_dim, float scale_log2,
            int causal, int dtype, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Split-KV first pass: per-(row, split) partial softmax statistics over key
 * chunk [s*ceil(seq_kv/splits), min((s+1)*ceil(seq_kv/splits), seq_kv)).
 * m_p, l_p: float32 (batch, num_heads, seq_q, splits) with strides p_strides4;
 * acc_p: float32 (batch, num_heads, seq_q, splits, head_dim), strides a_strides5.
 * m is in log2 units (already multiplied by scale_log2), l = sum exp2(s - m),
 * acc = sum exp2(s - m) v (unnormalised). An empty chunk gives (-inf, 0, 0).
 * Replaces gqa_split_first_kernel, gqa_kernels/gqa_split.py:26-112, launched at :168-183.
 */
int gqa_split_first(const void* q, const void* k, const void* v, float* m_p, float* l_p, float* acc_p,
                    const int64_t* q_strides4, const int64_t* k_strides4, const int64_t* v_strides4,
                    const int64_t* p_strides4, const int64_t* a_strides5, int batch, int num_heads,
                    int num_kv_heads, int seq_q, int seq_kv, int head_dim, float scale_log2, int causal,
                    int splits, int dtype, void* stream);

/*
 * Split-KV second pass: log-sum-exp combine of the partials above into O.
 * Replaces gqa_split_reduce_kernel, gqa_kernels/gqa_split.py:115-147, launched at :185-193.
 */
int gqa_split_reduce(const float* m_p, const float* l_p, const float* acc_p, void* o,
                     const int64_t* p_strides4, const int64_t* a_strides5, const int64_t* o_strides4,
                     int batch, int num_heads, int seq_q, int head_dim, int splits, int dtype, void* stream);

/*
 * One-launch split-KV forward: the key range is split into chunks sized for
 * the device's SM count and the last CTA of each (batch, kv_head, q-block)
 * combines the chunk partials in-kernel (atomic ticket, no second launch).
 * Same result as split_kv_forward, gqa_kernels/gqa_split.py:153-194.
 * The workspace must hold gqa_split_fused_workspace_bytes() bytes and its
 * ticket counters must be zero before the first call; every call leaves them
 * zero again. Calls sharing a workspace must be ordered on one stream.
 */
size_t gqa_split_fused_workspace_bytes(int batch, int num_heads, int num_kv_heads, int seq_q, int seq_kv,
                                       int head_dim);
int gqa_split_fused(const void* q, const void* k, const void* v, void* o, const int64_t* q_strides4,
                    const int64_t* k_strides4, const int64_t* v_strides4, const int64_t* o_strides4,
                    int batch, int num_heads, int num_kv_heads, int seq_q, int seq_kv, int head_dim,
                    float scale_log2, int causal, int dtype, void* workspace, size_t workspace_bytes,
                    void* stream);

/*
 * gqa_split_fused without a workspace argument, for callers that cannot
 * allocate device memory -- e.g. a host bound to this C ABI through an FFI
 * (Go, Java, Rust) that owns no CUDA allocator, or an engine that reserves all
 * of HBM for its own pool up front, where a cudaMalloc would fail or stall the
 * device in the middle of a decode step. The scratch lives in a static
 * __device__ array of GQA_NOALLOC_SCRATCH_BYTES that every GPU loading the
 * library holds until the process exits; the library calls no cudaMalloc,
 * cudaFree or allocating routine here. Problems whose scratch would exceed it
 * return GQA_ERR_SCRATCH_LIMIT (gqa_split_fused_workspace_bytes gives the
 * need). The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current; make that first call
 * before any stream capture. All calls share the one array: calls that
 * overlap on the GPU (other streams, other threads) race and must be ordered
 * by the caller. No counterpart in the reference.
 */
#define GQA_NOALLOC_SCRATCH_BYTES (4u << 20)
int gqa_split_fused_noalloc(const void* q, const void* k, const void* v, void* o, const int64_t* q_strides4,
                            const int64_t* k_strides4, const int64_t* v_strides4, const int64_t* o_strides4,
                            int batch, int num_heads, int num_kv_heads, int seq_q, int seq_kv, int head_dim,
                            float scale_log2, int causal, int dtype, void* stream);

/*
 * Partial attention over one shard of the key axis, for a key range split
 * across GPUs. k and v hold keys [kv_offset, kv_offset + seq_kv_local) of a
 * sequence of seq_kv_total keys; causal masking uses global key positions.
 * Outputs are float32, contiguous: m_out/l_out (batch, num_heads, seq_q),
 * acc_out (batch, num_heads, seq_q, head_dim), with the meaning of
 * gqa_split_first's (m, l, acc) for this shard. seq_kv_local may be 0 (a rank
 * whose share of the keys is empty): the outputs are then (-inf, 0, 0) for every
 * row, which gqa_lse_combine weighs 0, and k/v are not read.
 * No reference counterpart (the reference is single-GPU); the partial
 * definition follows gqa_kernels/gqa_split.py:102-112.
 */
size_t gqa_partial_workspace_bytes(int batch, int num_heads, int num_kv_heads, int seq_q, int seq_kv_local,
                                   int head_dim);
int gqa_partial(const void* q, const void* k, const void* v, float* m_out, float* l_out, float* acc_out,
                const int64_t* q_strides4, const int64_t* k_strides4, const int64_t* v_strides4, int batch,
                int num_heads, int num_kv_heads, int seq_q, int seq_kv_local, int kv_offset, int seq_kv_total,
                int head_dim, float scale_log2, int causal, int dtype, void* workspace, size_t workspace_bytes,
                void* stream);

/*
 * Log-sum-exp combine of `nparts` partial sets (e.g. one per GPU). Part s
 * holds, for row r = (b*num_heads + h)*seq_q + i, the values
 * m_parts[s*ml_part_stride + r], l_parts[s*ml_part_stride + r] and
 * acc_parts[s*acc_part_stride + r*head_dim + d] (float32), i.e. gqa_partial's
 * outputs stacked along a leading axis -- either as three stacked arrays or as
 * one packed [m | l | acc] buffer per part, as an all-gather produces.
 * Algebra of gqa_kernels/gqa_split.py:137-144, applied across parts.
 */
int gqa_lse_combine(const float* m_parts, const float* l_parts, const float* acc_parts, int nparts,
                    int64_t ml_part_stride, int64_t acc_part_stride, void* o, const int64_t* o_strides4, int batch,
                    int num_heads, int seq_q, int head_dim, int dtype, void* stream);

/*
 * Peer exchange: the key-sharded combine across the GPUs of one node without a
 * collective library. gqa_partial's outputs go straight from the partial kernel
 * into every rank's receive buffer (plain stores, over NVLink for the other
 * ranks), and each rank's combine waits for them in-kernel. It replaces
 * gqa_partial + an all-gather + gqa_lse_combine with two launches and no
 * collective call. No reference counterpart (the reference is single-GPU); the
 * algebra is gqa_kernels/gqa_split.py:137-144's across ranks.
 *
 * Each rank holds one exchange buffer (gqa_exchange_alloc, zeroed; it allocates
 * and synchronises, a setup call): [2 parities][nranks slots][slot_floats
 * floats] of packed partials [m | l | pad to 16 B | acc] (the layout of
 * gqa_lse_combine's packed form), then nranks uint64 counters (one per source
 * rank), then one uint64 call counter (the epoch). Every rank maps the other
 * ranks' buffers once: gqa_ipc_handle exports this process's buffer as a
 * GQA_IPC_HANDLE_BYTES handle, gqa_ipc_open maps another process's (CUDA IPC,
 * same node; never a multicast mapping), gqa_ipc_close unmaps it.
 *
 * Per call, on every rank, in this order on one stream:
 *   gqa_epoch_bump(epoch)       one thread: epoch += 1
 *   gqa_partial_peer(...)       writes this rank's partial into slot `rank`
 *                               of parity (epoch & 1) of every rank's buffer,
 *                               then adds 1 per unit to that rank's counter
 *                               for this source (system-scope release)
 *   gqa_lse_combine_peer(...)   waits (bounded) until every source's counter
 *                               reaches epoch x units, then combines into o
 * Every rank makes the same calls with the same shapes (so the epochs and unit
 * counts agree; gqa_partial_units gives the count), and every rank must hold at
 * least one key (seq_kv_local > 0; else GQA_ERR_UNSUPPORTED: use the all-gather
 * form, which accepts empty shards). Two parities let a rank start its next
 * call while another still reads this one: a rank cannot reach the call after
 * next before every rank has finished this call's combine. A source that never
 * arrives ends the combine's wait after the wait limit with GQA_ERR_TIMEOUT in
 * the device error word (gqa_device_error) and o unwritten.
 * peer_bases[i] / peer_cnts[i] are rank i's buffer and counters as this
 * process maps them (its own for i == rank); npeer <= 8.
 */
#define GQA_IPC_HANDLE_BYTES 64
int gqa_exchange_alloc(size_t bytes, void** ptr);
int gqa_exchange_free(void* ptr);
int gqa_ipc_handle(const void* ptr, void* handle);
int gqa_ipc_open(const void* handle, void** ptr);
int gqa_ipc_close(void* ptr);
int gqa_epoch_bump(unsigned long long* epoch, void* stream);
int gqa_partial_units(int batch, int num_heads, int num_kv_heads, int seq_q, int head_dim, int* units);
int gqa_partial_peer(const void* q, const void* k, const void* v, const int64_t* q_strides4, const int64_t* k_strides4,
                     const int64_t* v_strides4, int batch, int num_heads, int num_kv_heads, int seq_q,
                     int seq_kv_local, int kv_offset, int seq_kv_total, int head_dim, float scale_log2, int causal,
                     int dtype, float* const* peer_bases, unsigned long long* const* peer_cnts, int npeer, int rank,
                     const unsigned long long* epoch, int64_t slot_floats, int64_t parity_floats, void* workspace,
                     size_t workspace_bytes, void* stream);
int gqa_lse_combine_peer(const float* recv, const unsigned long long* cnt, const unsigned long long* epoch,
                         int nparts, int64_t slot_floats, int64_t parity_floats, int units, void* o,
                         const int64_t* o_strides4, int batch, int num_heads, int seq_q, int head_dim, int dtype,
                         void* stream);

/*
 * Paged decode: one new query token per sequence attends to that sequence's
 * cached keys, read from a paged K/V cache in the layout vLLM uses,
 * k_cache/v_cache (num_blocks, block_size, num_kv_heads, head_dim), contiguous.
 * Sequence b holds seq_lens[b] keys; its key k lives in physical block
 * block_table[b * bt_stride + k / block_size] at position k % block_size.
 * q/o are (num_seqs, num_heads, head_dim) with element strides q_strides3 /
 * o_strides3 (seq, head, d; d stride 1). block_size must be a power of two
 * >= 64; block_table and seq_lens are int32 device arrays; max_seq_len bounds
 * every seq_lens[b] and sizes the key split (the workspace query takes it).
 * A sequence with no key gives NaN, as the dense path does. The split
 * combine is fused into the launch when the workspace (zeroed before first
 * use; every call leaves it zero) holds gqa_paged_decode_workspace_bytes().
 * No reference counterpart: the reference's roadmap names a vLLM-shaped
 * interface (README.md:144); the attention is gqa_kernels/gqa_split.py's.
 */
size_t gqa_paged_decode_workspace_bytes(int num_seqs, int num_heads, int num_kv_heads, int max_seq_len,
                                        int head_dim);
int gqa_paged_decode(const void* q, const void* k_cache, const void* v_cache, void* o, const int64_t* q_strides3,
                     const int64_t* o_strides3, const int* block_table, int bt_stride, const int* seq_lens,
                     int num_seqs, int num_heads, int num_kv_heads, int head_dim, int block_size, int num_blocks,
                     int max_seq_len, float scale_log2, int dtype, void* workspace, size_t workspace_bytes,
                     void* stream);

/*
 * Paged forward (chunked prefill over a paged cache): each sequence's seq_q new
 * query tokens attend to its cached keys, read from the same vLLM-layout caches
 * as gqa_paged_decode. q/o are (num_seqs, num_heads, seq_q, head_dim) with
 * element strides q_strides / o_strides (the gqa_fwd convention). The queries
 * of sequence b are its last seq_q positions: with `causal`, query i sees keys
 * [0, seq_lens[b] - seq_q + i] (bottom-right alignment per sequence, the dense
 * path's rule); without, all seq_lens[b] keys. Rows that see no key give NaN.
 * Short chunks (group * seq_q <= 64) run the streaming kernel, longer ones the
 * tcgen05 prefill kernel, whose producer reads K/V tiles through the block
 * table. Cache slots past seq_lens[b] in a sequence's last block are read but
 * never reach O (their V rows are zeroed in shared memory before the PV MMA), so
 * stale or non-finite values there are harmless.
 * The key split is sized by max_seq_len; its workspace (zeroed before first
 * use; every call leaves it zero) is gqa_paged_fwd_workspace_bytes(). Called
 * with seq_q = 1 and causal = 0 this is gqa_paged_decode.
 * No reference counterpart: the roadmap's vLLM-shaped interface (README.md:144)
 * over the attention of gqa_kernels/gqa_fwd.py.
 */
size_t gqa_paged_fwd_workspace_bytes(int num_seqs, int num_heads, int num_kv_heads, int seq_q, int max_seq_len,
                                     int head_dim);
int gqa_paged_fwd(const void* q, const void* k_cache, const void* v_cache, void* o, const int64_t* q_strides,
                  const int64_t* o_strides, const int* block_table, int bt_stride, const int* seq_lens,
                  int num_seqs, int num_heads, int num_kv_heads, int seq_q, int head_dim, int block_size,
                  int num_blocks, int max_seq_len, float scale_log2, int causal, int dtype, void* workspace,
                  size_t workspace_bytes, void* stream);

/*
 * gqa_paged_fwd over fp8 caches: k_cache/v_cache hold e4m3 values (one byte
 * each, same layout), and key = stored key x k_scale, value = stored value x
 * v_scale (vLLM's fp8 KV-cache convention; both scales > 0). q/o keep `dtype`
 * (bf16 or fp16). head_dim must be 128 and group * seq_q <= 64 (decode and
 * short chunks: the streaming kernel, whose K/V fragments are converted exactly
 * from e4m3 to f16 in registers; both MMAs run in f16, so |q| must stay within
 * the f16 range). Otherwise GQA_ERR_UNSUPPORTED. The workspace is
 * gqa_paged_fwd_workspace_bytes(). Halves the bytes streamed per key against
 * 16-bit caches.
 * No reference counterpart: the reference's K/V are bf16 or fp16 only.
 */
int gqa_paged_fwd_kv8(const void* q, const void* k_cache, const void* v_cache, void* o, const int64_t* q_strides,
                      const int64_t* o_strides, const int* block_table, int bt_stride, const int* seq_lens,
                      int num_seqs, int num_heads, int num_kv_heads, int seq_q, int head_dim, int block_size,
                      int num_blocks, int max_seq_len, float scale_log2, float k_scale, float v_scale, int causal,
                      int dtype, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Cache write of the paged interface (vLLM's reshape_and_cache_flash): token t's K
 * and V rows, key/value (num_tokens, num_kv_heads, head_dim) with element strides
 * k_strides3 / v_strides3 (d stride 1, the others multiples of 8 elements), go to
 * slot slot_mapping[t] (int64; block = slot / block_size, position = slot %
 * block_size) of the (num_blocks, block_size, num_kv_heads, head_dim) caches. A
 * negative slot is a padding token and is skipped. 16-bit caches (dtype) receive the
 * rows unchanged; with cache_fp8 the caches are e4m3 and receive x / k_scale (x /
 * v_scale) rounded to nearest even and saturated to +-448, vLLM's convention (real
 * value = stored value x scale; scales > 0). A slot >= num_blocks * block_size is not
 * written: its row is skipped and GQA_ERR_INVALID_ARG is recorded in the device error
 * word (site 201; gqa_device_error). Tokens must map to distinct slots.
 * No reference counterpart: the cache-write half of the roadmap's vLLM-shaped
 * interface (README.md:144).
 */
int gqa_paged_kv_append(const void* key, const void* value, const int64_t* k_strides3, const int64_t* v_strides3,
                        void* k_cache, void* v_cache, const int64_t* slot_mapping, int num_tokens, int num_kv_heads,
                        int head_dim, int block_size, int num_blocks, int dtype, int cache_fp8, float k_scale,
                        float v_scale, void* stream);

/*
 * The tcgen05 prefill path's launch plan for a shape on `sm_count` SMs, without
 * launching (host only; needs no GPU). plan[0..4] = units (query pairs x batch x
 * kv heads), nsplit (CTAs per unit; > 1 when the units are fewer than the SMs),
 * key tiles per split, head-major unit order (0/1), grid size.
 * No reference counterpart (the reference launches one program per query block).
 */
int gqa_prefill_plan(int batch, int num_heads, int num_kv_heads, int seq_q, int seq_kv, int head_dim, int causal,
                     int sm_count, int* plan);

/*
 * Reads (and clears, if `clear` is nonzero) the device error word of the
 * current device: 0, or GQA_ERR_TIMEOUT when a bounded in-kernel wait expired.
 * `site` (optional) receives the wait site id. Synchronises the current device.
 * No reference counterpart (the reference has no in-kernel waits).
 */
int gqa_device_error(int* code, int* site, int clear);

/* Number of SMs of the current device as used for split sizing. */
int gqa_sm_count(void);

/*
 * Test hooks of the checked build (libgqa_sm100_debug.so, build.py --debug); the
 * release library returns GQA_ERR_UNSUPPORTED from both. No reference counterpart:
 * they exist to test this library's failure detection and arithmetic on the GPU.
 *
 * gqa_debug_inject: the TMA producer of CTA `cta` withholds its load number `load`
 * (prefill: the K/V tile load index, K and V alternating; streaming kernel: the
 * stage index) in every following launch, and every bounded in-kernel wait gives up
 * after wait_limit_ns (<= 0 restores the default). The consumer's wait on the
 * withheld load then expires: the kernel records GQA_ERR_TIMEOUT in the device error
 * word, aborts the CTA (its other waits end, issued copies land, TMEM is freed) and
 * returns. cta = -1 withholds nothing. Applies to the current device.
 *
 * gqa_debug_exp2_poly2: y[i] = the kernels' FMA-pipe exp2 (the polynomial the prefill
 * softmax uses for one column pair in eight) of x[i], for i < n; device pointers.
 */
int gqa_debug_inject(int cta, int load, long long wait_limit_ns);
int gqa_debug_exp2_poly2(const float* x, float* y, int n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GQA_SM100_H_ */
