/*
 * akt.h — C ABI of the B200 (sm_100a) attention kernels.
 *
 * Plain C: device pointers, element strides and sizes; no torch types.  Every
 * entry point is asynchronous on the given CUDA stream (a cudaStream_t passed
 * as void*, NULL = legacy default stream), never synchronises the host, and
 * returns an akt_status.  On a non-zero return akt_last_error() gives a
 * message for the calling thread.
 *
 * Each entry point replaces the Triton launcher of one reference module of
 * KiritoHugh/attention_kernel_triton (cited per function).  Tensor shapes and
 * argument meanings are those of the reference launchers; strides are in
 * elements.  Out-of-range page ids or token indices never fault: the kernel
 * skips the access and records a code in the device status word
 * (akt_device_status).
 *
 * Entry points that need scratch take a caller-owned device workspace whose
 * size the matching *_workspace_size() function returns for the same args.
 */
#ifndef AKT_H_
#define AKT_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AKT_ABI_VERSION 1

typedef enum akt_status {
  AKT_OK = 0,
  AKT_ERR_INVALID = 1,     /* bad shape / argument (the reference asserts) */
  AKT_ERR_UNSUPPORTED = 2, /* layout the kernel cannot take (caller may copy to contiguous) */
  AKT_ERR_CUDA = 3,        /* CUDA runtime error (launch, attribute) */
  AKT_ERR_WORKSPACE = 4    /* workspace missing or too small */
} akt_status;

typedef enum akt_dtype { AKT_FLOAT16 = 0, AKT_BFLOAT16 = 1 } akt_dtype;

/* ------------------------------------------------------------------------ */
/* library / device status                                                  */
/* ------------------------------------------------------------------------ */
int akt_abi_version(void);
const char* akt_last_error(void);
/* First error code any kernel recorded on `device` since the last clear
 * (0 = none; 1 wait timeout, 2 page id out of pool, 3 token index out of
 * sequence, 4 malformed indptr, 5 kept-index list longer than its buffer).
 * Synchronises that device. */
int akt_device_status(int device, unsigned int* status_out);
int akt_clear_device_status(int device);

/* Benchmark hook: while enabled on the calling thread, each entry point
 * records a CUDA event pair around its main kernel on the launch stream.
 * akt_profile_read waits for them, returns the summed device milliseconds
 * and the number of timed launches, and resets the record. */
int akt_profile_enable(int on);
int akt_profile_read(double* total_ms, int64_t* launches);

/* ------------------------------------------------------------------------ */
/* causal / non-causal GQA prefill, optionally padded var-len               */
/* replaces flash_attention_prefill(Q, K, V, causal, softmax_scale,         */
/*   GQA_group_size) of prefill_flash_attention.py:342-383 and              */
/*   flash_attention_prefill(..., varlen) of                                */
/*   prefill_flash_attention_var_len_padding.py:348-391                     */
/* Q/O [batch, num_qo_heads, seq_len, head_dim], K/V [batch, num_kv_heads,  */
/* seq_len, head_dim]; kv head of qo head h is h / (num_qo_heads /          */
/* num_kv_heads); causal is top-left aligned (row i sees keys j <= i).      */
/* varlen (int32 [batch], or NULL): rows i >= varlen[b] are written as      */
/* zeros; keys are not masked by varlen (as in the reference).  head_dim 64 */
/* or 128; no workspace.                                                    */
/* ------------------------------------------------------------------------ */
typedef struct akt_prefill_args {
  const void* q;
  int64_t q_stride_batch, q_stride_head, q_stride_token, q_stride_dim;
  const void* k;
  int64_t k_stride_batch, k_stride_head, k_stride_token, k_stride_dim;
  const void* v;
  int64_t v_stride_batch, v_stride_head, v_stride_token, v_stride_dim;
  void* out;
  int64_t out_stride_batch, out_stride_head, out_stride_token, out_stride_dim;
  const int32_t* varlen;
  int32_t batch, num_qo_heads, num_kv_heads, seq_len, head_dim;
  int32_t causal;
  int32_t dtype;
  float softmax_scale;
} akt_prefill_args;

int akt_prefill(const akt_prefill_args* args, void* stream);

/* akt_prefill that also writes each row's natural-log sum-exp of the scaled   */
/* scores over its visible keys, lse [batch, num_qo_heads, seq_len] fp32      */
/* (token stride 1; -inf for var-len padding rows).  The reference computes  */
/* this value and leaves its store commented out                             */
/* (prefill_flash_attention.py:331-334: tmp_m_i += tl.math.log(tmp_l_i)).    */
int akt_prefill_with_lse(const akt_prefill_args* args, float* lse, int64_t lse_stride_batch,
                         int64_t lse_stride_head, void* stream);

/* ------------------------------------------------------------------------ */
/* dense ("redundant") GQA decode                                           */
/* replaces flash_attention_decode(q, K, V, softmax_scale, GQA_group_size)  */
/* decode_flash_attention_redundant.py:233-271                              */
/* ------------------------------------------------------------------------ */
typedef struct akt_decode_dense_args {
  const void* q; /* [batch, num_qo_heads, 1, head_dim] */
  int64_t q_stride_batch, q_stride_head, q_stride_dim;
  const void* k; /* [batch, num_kv_heads, seq_len, head_dim] */
  int64_t k_stride_batch, k_stride_head, k_stride_token, k_stride_dim;
  const void* v; /* [batch, num_kv_heads, seq_len, head_dim] */
  int64_t v_stride_batch, v_stride_head, v_stride_token, v_stride_dim;
  void* out; /* [batch, num_qo_heads, 1, head_dim] */
  int64_t out_stride_batch, out_stride_head, out_stride_dim;
  int32_t batch, num_qo_heads, num_kv_heads, seq_len, head_dim;
  int32_t dtype; /* akt_dtype of q, k, v and out */
  float softmax_scale;
} akt_decode_dense_args;

size_t akt_decode_dense_workspace_size(const akt_decode_dense_args* args);
int akt_decode_dense(const akt_decode_dense_args* args, void* workspace, size_t workspace_bytes,
                     void* stream);

/* ------------------------------------------------------------------------ */
/* paged var-len GQA decode                                                 */
/* replaces flash_attention_decode_paged(q, paged_kv_cache, kv_page_indptr, */
/*   kv_page_indices, kv_last_page_len)                                     */
/* decode_flash_attention_redundant_var_len_paged.py:228-274                */
/* Sequence b is pages kv_page_indices[indptr[b] .. indptr[b+1]); its last  */
/* page holds kv_last_page_len[b] tokens (clamped to [0, page_size]); an    */
/* empty sequence yields zeros.  softmax_scale is 1/sqrt(head_dim) in the   */
/* reference (line 244); it is an argument here.                            */
/* ------------------------------------------------------------------------ */
typedef struct akt_decode_paged_args {
  const void* q; /* [batch, num_qo_heads, 1, head_dim] */
  int64_t q_stride_batch, q_stride_head, q_stride_dim;
  const void* kv_cache; /* [num_pages, 2, num_kv_heads, page_size, head_dim] */
  int64_t kv_stride_page, kv_stride_kv, kv_stride_head, kv_stride_token, kv_stride_dim;
  int64_t num_pages;               /* extent of kv_cache dim 0 (bounds check) */
  const int32_t* kv_page_indptr;   /* [batch + 1] */
  const int32_t* kv_page_indices;  /* [num_page_entries] */
  const int32_t* kv_last_page_len; /* [batch] */
  int64_t num_page_entries;
  void* out; /* [batch, num_qo_heads, head_dim] */
  int64_t out_stride_batch, out_stride_head, out_stride_dim;
  int32_t batch, num_qo_heads, num_kv_heads, page_size, head_dim;
  int32_t dtype;
  float softmax_scale;
} akt_decode_paged_args;

size_t akt_decode_paged_workspace_size(const akt_decode_paged_args* args);
int akt_decode_paged(const akt_decode_paged_args* args, void* workspace, size_t workspace_bytes,
                     void* stream);

/* Allocation-free paged decode.  No counterpart in the reference: it exists for
 * callers that cannot allocate device memory when they run the decode (plugin
 * hosts that pass only input and output buffers, runtimes that forbid
 * cudaMalloc after start-up).  Same arguments, semantics and kernels as
 * akt_decode_paged, but the split-KV scratch lives in a fixed 16 MiB array
 * owned by the library (held on every GPU that loads the library, until
 * process exit); nothing is allocated per call.  A call whose partials would
 * not fit returns AKT_ERR_WORKSPACE with the size it needed.  The first call
 * on a device looks up that array's device address (set-up, once per device,
 * with the target device current); make that first call before any stream
 * capture.  The address is looked up again when the context current at a
 * call differs from the one it was found under (a driver-API caller with its
 * own context); a device reset (cudaDeviceReset) is not detected, so a
 * process must not call this entry point on a device after resetting it.
 * All calls share the array and it keeps the last call's contents (nothing in
 * it needs to start at zero): calls that overlap on the GPU, on any streams,
 * race and must not be issued. */
int akt_decode_paged_noalloc(const akt_decode_paged_args* args, void* stream);

/* ------------------------------------------------------------------------ */
/* sparse-token GQA decode, dense KV                                        */
/* replaces sparsetoken_flash_attention_decode(q, K, V, sparse_ind,         */
/*   sparse_nnz, softmax_scale, GQA_group_size)                             */
/* sparsetoken_decode_flash_attention_redundant.py:127-170                  */
/* Head h of batch b attends to tokens sparse_ind[b, h, 0:nnz) of its kv    */
/* head; nnz <= 0 yields zeros.  Token indices outside [0, seq_len) are     */
/* skipped and recorded in the device status word.                          */
/* ------------------------------------------------------------------------ */
typedef struct akt_sparse_dense_args {
  const void* q; /* [batch, num_qo_heads, 1, head_dim] */
  int64_t q_stride_batch, q_stride_head, q_stride_dim;
  const void* k; /* [batch, num_kv_heads, seq_len, head_dim] */
  int64_t k_stride_batch, k_stride_head, k_stride_token, k_stride_dim;
  const void* v;
  int64_t v_stride_batch, v_stride_head, v_stride_token, v_stride_dim;
  const int32_t* sparse_ind; /* [batch, num_qo_heads, max_nnz], -1 padded */
  int64_t ind_stride_batch, ind_stride_head, ind_stride_pos;
  const int32_t* sparse_nnz; /* [batch, num_qo_heads(, 1)] */
  int64_t nnz_stride_batch, nnz_stride_head;
  void* out; /* [batch, num_qo_heads, 1, head_dim] */
  int64_t out_stride_batch, out_stride_head, out_stride_dim;
  int32_t batch, num_qo_heads, num_kv_heads, seq_len, head_dim, max_nnz;
  int32_t dtype;
  float softmax_scale;
} akt_sparse_dense_args;

size_t akt_sparse_dense_workspace_size(const akt_sparse_dense_args* args);
int akt_sparse_dense(const akt_sparse_dense_args* args, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* sparse-token GQA decode, paged KV (and the MagicPIG variant)             */
/* replaces sparsetoken_flash_attention_decode_paged(q, paged_kv_cache,     */
/*   kv_page_indptr, kv_page_indices, sparse_ind, sparse_nnz)               */
/* sparsetoken_decode_flash_attention_redundant_var_len_paged.py:170-232    */
/* Kept token t of sequence b is row t % page_size of physical page         */
/* kv_page_indices[indptr[b] + t / page_size]; tokens past the sequence's   */
/* page list are skipped and recorded.  nnz <= 0 yields zeros.              */
/* ------------------------------------------------------------------------ */
typedef struct akt_sparse_paged_args {
  const void* q; /* [batch, num_qo_heads, 1, head_dim] */
  int64_t q_stride_batch, q_stride_head, q_stride_dim;
  const void* kv_cache; /* [num_pages, 2, num_kv_heads, page_size, head_dim] */
  int64_t kv_stride_page, kv_stride_kv, kv_stride_head, kv_stride_token, kv_stride_dim;
  int64_t num_pages;
  const int32_t* kv_page_indptr;  /* [batch + 1] */
  const int32_t* kv_page_indices; /* [num_page_entries] */
  int64_t num_page_entries;
  const int32_t* sparse_ind; /* [batch, num_qo_heads, max_nnz] */
  int64_t ind_stride_batch, ind_stride_head, ind_stride_pos;
  const int32_t* sparse_nnz; /* [batch, num_qo_heads(, 1)] */
  int64_t nnz_stride_batch, nnz_stride_head;
  /* MagicPIG only (NULL otherwise): per-(batch, qo head) LSH parameters K, L (fp32) */
  const float* magicpig_k;
  const float* magicpig_l;
  int64_t param_stride_batch, param_stride_head;
  void* out; /* [batch, num_qo_heads, head_dim] */
  int64_t out_stride_batch, out_stride_head, out_stride_dim;
  int32_t batch, num_qo_heads, num_kv_heads, page_size, head_dim, max_nnz;
  int32_t dtype;
  float softmax_scale; /* ignored by the MagicPIG entry point (fixed 1/sqrt(head_dim)) */
} akt_sparse_paged_args;

size_t akt_sparse_paged_workspace_size(const akt_sparse_paged_args* args);
int akt_sparse_paged(const akt_sparse_paged_args* args, void* workspace, size_t workspace_bytes, void* stream);

/* MagicPIG sparse-token paged decode with norm                              */
/* replaces magicpig_sparsetoken_flash_attention_decode_paged(q,             */
/*   paged_kv_cache, kv_page_indptr, kv_page_indices, sparse_ind,            */
/*   sparse_nnz, K, L)                                                       */
/* magicpig_sparsetoken_decode_flash_attention_redundant_var_len_paged_      */
/*   with_norm.py:166-209: score_i = q.k_i/sqrt(D) - log(u_i),               */
/*   u_i = 1 - (1-p^K)^L - L p^K (1-p^K)^(L-1), p = 1 - acos(cos(q,k_i))/pi  */
/*   (clamps as in that file's naive reference, lines 263-278).              */
size_t akt_magicpig_paged_workspace_size(const akt_sparse_paged_args* args);
int akt_magicpig_paged(const akt_sparse_paged_args* args, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* sparse-token decodes with CSR kept-index lists                           */
/* The "inds + ptr" index format proposed in the reference's notes          */
/* (sparse_decode_flash_attention.py:13-15), which has no implementation    */
/* there: the kept tokens of (batch b, qo head h) are                       */
/* args->sparse_ind[sparse_ptr[r] .. sparse_ptr[r + 1]) with                */
/* r = b * num_qo_heads + h, so lists are not padded to a common length.    */
/* sparse_ptr holds batch * num_qo_heads + 1 offsets into a flat array of   */
/* num_inds entries; args->sparse_nnz and the ind strides are not read;     */
/* args->max_nnz bounds every row's length (it sizes the workspace, as      */
/* *_workspace_size reports for the same args; longer rows are cut there   */
/* and recorded, status 3).  Rows with malformed offsets keep nothing and   */
/* are recorded (status 4).  Same kernels and semantics otherwise.          */
/* ------------------------------------------------------------------------ */
int akt_sparse_dense_csr(const akt_sparse_dense_args* args, const int32_t* sparse_ptr, int64_t num_inds,
                         void* workspace, size_t workspace_bytes, void* stream);
int akt_sparse_paged_csr(const akt_sparse_paged_args* args, const int32_t* sparse_ptr, int64_t num_inds,
                         void* workspace, size_t workspace_bytes, void* stream);
int akt_magicpig_paged_csr(const akt_sparse_paged_args* args, const int32_t* sparse_ptr, int64_t num_inds,
                           void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* KV split across devices (long single-sequence sparse decode)             */
/* No reference counterpart (the reference keeps no LSE; its store is       */
/* commented out at prefill_flash_attention.py:331-334).  The *_partial     */
/* entry points run the matching sparse decode over this device's tokens    */
/* and, instead of the typed output, write the fp32 output normalised over  */
/* those tokens, o_part [batch, num_qo_heads, head_dim], and its natural-   */
/* log sum-exp, lse_part [batch, num_qo_heads] (-inf where no token was     */
/* kept).  akt_lse_merge combines num_parts such partials into out rows of  */
/* head_dim elements (row stride out_row_stride); part i's O starts at      */
/* o_parts + i * o_part_stride and its LSE at lse_parts + i *               */
/* lse_part_stride (floats), so one all-gathered [O | LSE] buffer per       */
/* device merges in place.                                                  */
/* ------------------------------------------------------------------------ */
int akt_sparse_dense_partial(const akt_sparse_dense_args* args, float* o_part, float* lse_part, void* workspace,
                             size_t workspace_bytes, void* stream);
int akt_sparse_paged_partial(const akt_sparse_paged_args* args, float* o_part, float* lse_part, void* workspace,
                             size_t workspace_bytes, void* stream);
int akt_magicpig_paged_partial(const akt_sparse_paged_args* args, float* o_part, float* lse_part,
                               void* workspace, size_t workspace_bytes, void* stream);
int akt_lse_merge(const float* o_parts, int64_t o_part_stride, const float* lse_parts, int64_t lse_part_stride,
                  int32_t num_parts, int64_t rows, int32_t head_dim, void* out, int64_t out_row_stride,
                  int32_t dtype, void* stream);

/* ------------------------------------------------------------------------ */
/* KV split with the exchange fused into the kernels (NVLink peer stores)   */
/* instead of a library all-gather.  Each device owns one exchange region   */
/* (akt_ipc_alloc: cudaMalloc'd, zeroed, exported as a CUDA IPC handle that */
/* the other processes map with akt_ipc_open).  Per call (epoch e = 1, 2,   */
/* ...; parity e & 1 selects one of two buffers so a writer never reaches a */
/* slot its reader may still be reading):                                   */
/*  - akt_sparse_dense_partial_peer runs the sparse decode over this        */
/*    device's tokens and its last kernel stores the fp32 partial           */
/*    [O (rows x head_dim) | LSE (rows)] into slot `rank` of every device's */
/*    data area with plain stores, then, once all its CTAs are done, writes */
/*    e into flag `rank` of every device (system-scope release);            */
/*  - akt_lse_merge_peer waits (bounded: 2 s, then status 1 and zeros)      */
/*    until this device's flags all read e, merges its data area, and its   */
/*    last CTA clears those flags, so flag values need not grow and a       */
/*    captured graph per parity can be replayed.                            */
/* Only plain stores and loads touch peer memory.  peer_data[r] / peer_flags[r] */
/* are device r's data area / flag array for this call's parity, as mapped  */
/* in the calling process; counter is this device's completion counter.     */
/* ------------------------------------------------------------------------ */
#define AKT_MAX_PEERS 8

typedef struct akt_peer_exchange {
  float* peer_data[AKT_MAX_PEERS];     /* [world][rows * head_dim + rows] fp32 each */
  uint32_t* peer_flags[AKT_MAX_PEERS]; /* [world] each */
  uint32_t* counter;                   /* this device: CTAs of the publishing kernel done */
  uint32_t* merge_counter;             /* this device: CTAs of the merge done */
  int32_t world, rank;
  uint32_t epoch;                      /* any non-zero value, the same on every rank */
} akt_peer_exchange;

int akt_ipc_alloc(size_t bytes, void** dev_ptr, void* handle_out /* 64 bytes */);
int akt_ipc_open(const void* handle /* 64 bytes */, void** dev_ptr);
int akt_ipc_close(void* dev_ptr);
int akt_ipc_free(void* dev_ptr);
int akt_sparse_dense_partial_peer(const akt_sparse_dense_args* args, const akt_peer_exchange* x, void* workspace,
                                  size_t workspace_bytes, void* stream);
int akt_lse_merge_peer(const akt_peer_exchange* x, int64_t rows, int32_t head_dim, void* out, int64_t out_row_stride,
                       int32_t dtype, void* stream);
/* The two calls above in one: the sparse decode over this device's tokens,  */
/* the publication of its partial and, in the same merge kernel, the wait    */
/* for every rank's flag and the final merge into args->out (strides of      */
/* args).  Two launches per step instead of three.  The merge grid (one CTA  */
/* per (batch, unit)) waits on itself, so calls with more (batch, unit)      */
/* pairs than four per SM return AKT_ERR_UNSUPPORTED (use the pair above).   */
int akt_sparse_dense_split_peer(const akt_sparse_dense_args* args, const akt_peer_exchange* x, void* workspace,
                                size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* paged KV cache append (write path; no reference counterpart: the         */
/* reference builds its pools in Python, decode_flash_attention_redundant_  */
/* var_len_paged.py:337-353)                                                 */
/* The page table (same CSR format as the paged decodes) already covers the */
/* appended tokens: sequence b holds len_b = (pages_b - 1) * page_size +    */
/* kv_last_page_len[b] tokens after the append, the last n_b =              */
/* append_indptr[b+1] - append_indptr[b] of them new.  Appended row i of    */
/* sequence b (row append_indptr[b] + i of append_k / append_v, each        */
/* [num_append, num_kv_heads, head_dim]) is written at position             */
/* len_b - n_b + i.  Bad page ids / positions / indptrs are skipped and     */
/* recorded (status 2 / 3 / 4).  No workspace.                              */
/* ------------------------------------------------------------------------ */
typedef struct akt_append_paged_args {
  void* kv_cache; /* [num_pages, 2, num_kv_heads, page_size, head_dim] */
  int64_t kv_stride_page, kv_stride_kv, kv_stride_head, kv_stride_token, kv_stride_dim;
  int64_t num_pages;
  const int32_t* kv_page_indptr;   /* [batch + 1] */
  const int32_t* kv_page_indices;  /* [num_page_entries] */
  const int32_t* kv_last_page_len; /* [batch], after the append */
  int64_t num_page_entries;
  const void* append_k; /* [num_append, num_kv_heads, head_dim] */
  int64_t k_stride_token, k_stride_head, k_stride_dim;
  const void* append_v;
  int64_t v_stride_token, v_stride_head, v_stride_dim;
  const int32_t* append_indptr; /* [batch + 1] */
  int64_t num_append;
  int32_t batch, num_kv_heads, page_size, head_dim, dtype;
} akt_append_paged_args;

int akt_append_paged_kv(const akt_append_paged_args* args, void* stream);

/* ------------------------------------------------------------------------ */
/* keep mask <-> padded kept-index lists, on the device                     */
/* replaces the Python loops of                                             */
/* sparsetoken_decode_flash_attention_redundant.py:283-295 (a per-token     */
/* keep mask to sparse_ind / sparse_nnz) and :317-324 (the lists back to    */
/* precompute_mask); the reference has no library function for either.     */
/* mask -> lists: kept positions ascending, the rest of each list -1; an    */
/* empty mask keeps token 0 when keep_first_if_empty (the reference's       */
/* rule); more than max_kept kept tokens keeps the first max_kept and       */
/* records status 5.  lists -> mask: nnz 0 reads as 1, entries are Python   */
/* indices (negative counts from the end, so -1 padding marks the last      */
/* token, as the reference loop does); entries outside [-seq_len, seq_len)  */
/* are skipped and recorded (status 3).  Masks are bytes (torch.bool), one  */
/* per token, token stride 1; lists have position stride 1.                 */
/* ------------------------------------------------------------------------ */
typedef struct akt_mask_to_index_args {
  const uint8_t* mask; /* [batch, num_heads, seq_len] */
  int64_t mask_stride_batch, mask_stride_head;
  int32_t* sparse_ind; /* [batch, num_heads, max_kept] (output) */
  int64_t ind_stride_batch, ind_stride_head;
  int32_t* sparse_nnz; /* [batch, num_heads(, 1)] (output) */
  int64_t nnz_stride_batch, nnz_stride_head;
  int32_t batch, num_heads, seq_len, max_kept;
  int32_t keep_first_if_empty;
} akt_mask_to_index_args;

int akt_mask_to_sparse_index(const akt_mask_to_index_args* args, void* stream);

typedef struct akt_index_to_mask_args {
  const int32_t* sparse_ind; /* [batch, num_heads, max_kept] */
  int64_t ind_stride_batch, ind_stride_head;
  const int32_t* sparse_nnz; /* [batch, num_heads(, 1)] */
  int64_t nnz_stride_batch, nnz_stride_head;
  uint8_t* mask; /* [batch, num_heads, seq_len] (output) */
  int64_t mask_stride_batch, mask_stride_head;
  int32_t batch, num_heads, seq_len, max_kept;
} akt_index_to_mask_args;

int akt_sparse_index_to_mask(const akt_index_to_mask_args* args, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* AKT_H_ */
