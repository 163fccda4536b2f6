/*
 * drinkme_b200 — the C ABI of the B200-native radix decode + linear hot path.
 *
 * Every entry point returns 0 on success and a nonzero status on failure,
 * writing a NUL-terminated message into (err, err_len) when err_len > 0 —
 * the convention of the reference's one native entry point
 * (src/drinkme/codec/radix_native.cpp:211-236, `radix_native(op, ...,
 * char* error, uint64_t error_size)`). No entry point takes a torch type:
 * pointers, sizes and a `void* stream` (a cudaStream_t; NULL = the legacy
 * default stream).
 *
 * Pointer residency: arrays named `host_*` are host memory; every other
 * array argument is device memory on the tensor's device. Calls that take a
 * stream enqueue work on it and return without synchronising (CUDA-graph
 * capturable), except where noted.
 *
 * Status codes: DM_OK 0, DM_EINVAL 1 (bad argument / malformed pack),
 * DM_ECUDA 2 (a CUDA API error), DM_EDEVICE 3 (a kernel reported a device
 * error, e.g. a bounded wait that gave up), DM_ENOMEM 4.
 */
#ifndef DRINKME_B200_H
#define DRINKME_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DM_OK 0
#define DM_EINVAL 1
#define DM_ECUDA 2
#define DM_EDEVICE 3
#define DM_ENOMEM 4

/* element types of activations and outputs */
#define DM_BF16 0
#define DM_F32 1

/* The widest activation batch one GEMV call serves: the reference's
 * MC_MAX (src/drinkme/codec/ops.py:19), the structural cap of the
 * multi-column kernel (radix_ops.py:379-398 refuses M outside 1..8). */
#define DM_MC_MAX 8

/* The most ranks (GPUs of one box) a row-sharded linear gathers over. */
#define DM_MAX_RANKS 8

typedef struct dm_tensor dm_tensor; /* opaque device-resident radix tensor */

typedef struct dm_tensor_info {
    int64_t R, C;              /* the full tensor's shape */
    int64_t row_begin, rows;   /* the shard this handle holds: rows [row_begin, row_begin + rows) */
    int32_t block_size, nwidths;
    int32_t widths[8];
    int64_t nblocks;           /* rows * ceil(C / block_size) */
    int64_t payload_words;     /* NW: the pack payload words of this shard */
    int64_t read_bytes;        /* radix_ops.read_bytes of this shard: NW*4 + directory + tables + schedule */
    int64_t resident_bytes;    /* device bytes the handle holds (layout + scratch) */
    int32_t fast_path;         /* 1 when the sm_100a sip kernel serves this tensor's GEMV */
    int32_t device;
    int64_t device_bytes_per_call; /* read_bytes' count over what the kernels stream: differs when the
                                      loader re-encoded a non-sip pack as sip (dm_tensor_create) */
    uint64_t layout_ptr;       /* the device address of the B200 layout the kernels stream (read only) */
    int64_t layout_bytes;      /* its size: the unit-major payload and the zero tail pad */
} dm_tensor_info;

/* Library version (major * 10000 + minor * 100 + patch). */
int dm_version(void);

/* Load one pack-format-1 radix tensor onto `device`, rows [row_begin,
 * row_end) of it (the whole tensor: 0, R). Replaces
 * swap.to_device_radix (src/drinkme/codec/swap.py:80-161) for the device
 * side: it validates the descriptors as radix.validate does
 * (src/drinkme/codec/radix.py:174-238; same messages), then lays the
 * shard's blocks out for the B200 kernels (unit-major, 16-byte aligned,
 * per-unit headers, the gulp schedule and, for the sip fast path, an
 * escape index) and copies it to the device. Host pointers: the pack's
 * rx_palette (unpadded, `npalette` entries), rx_offsets (R*NB+1 entries),
 * rx_data (`nwords`). Synchronous. A pack of another profile (gulp,
 * balanced) with 1024-weight blocks and rows of whole blocks is decoded on
 * the host and re-encoded as sip for the sip kernels (the same bits; the
 * handle still reports the pack's own widths, payload words and read_bytes;
 * device_bytes_per_call gives the re-encoded count). */
int dm_tensor_create(const uint8_t *host_palette, size_t npalette, const uint32_t *host_offsets,
                     size_t noffsets, const uint32_t *host_data, size_t nwords, int64_t R, int64_t C,
                     const int32_t *host_widths, int32_t nwidths, int32_t block_size, int64_t row_begin,
                     int64_t row_end, int32_t device, dm_tensor **out, char *err, size_t err_len);

/* One pack-format-1 tensor (or row range of one) for dm_tensor_create_multi:
 * the arguments of dm_tensor_create, gathered. */
typedef struct dm_pack_part {
    const uint8_t *host_palette;
    size_t npalette;
    const uint32_t *host_offsets;
    size_t noffsets;
    const uint32_t *host_data;
    size_t nwords;
    int64_t R, C;
    const int32_t *host_widths;
    int32_t nwidths, block_size;
    int64_t row_begin, row_end;
} dm_pack_part;

/* A FUSED tensor: the rows of `nparts` packs that read the same activations
 * (q, k and v; gate and up) stacked in order into one handle, so one GEMV
 * launch computes [y_0 | y_1 | ...] = x @ [W_0; W_1; ...]^T. Each part is
 * validated as dm_tensor_create validates it and keeps its own palette
 * (its exponent tables ride in the unit headers). Every part must be sip
 * (widths 3, 8) with 1024-weight blocks, all share C (a multiple of 1024),
 * and every part but the last must contribute a multiple of 16 rows
 * (DM_EINVAL otherwise). The handle's R and rows are the total rows; its
 * read_bytes the parts' sum. No reference counterpart: the reference runs
 * one RadixCompressedLinear per projection (src/drinkme/codec/swap.py:
 * 395-456); the fused handle serves the same arithmetic in one launch. */
int dm_tensor_create_multi(const dm_pack_part *parts, int32_t nparts, int32_t device, dm_tensor **out, char *err,
                           size_t err_len);

int dm_tensor_destroy(dm_tensor *t);

/* A second handle holding a device-side copy of `src` (same device, its own
 * buffers and scratch): loads one packed tensor into several places in HBM
 * without repeating the host layout. No reference counterpart (the
 * reference builds every resident tensor from its pack: swap.py:80-161). */
int dm_tensor_clone(const dm_tensor *src, dm_tensor **out, char *err, size_t err_len);

int dm_tensor_get_info(const dm_tensor *t, dm_tensor_info *info);

/* y[M, rows] = x[M, C] @ W[rows, C]^T (+ bias), fp32 accumulate, the bias
 * added in fp32 and ONE rounding to `out_dtype`. Replaces
 * radix_ops.gemv_fused / gemv / gemv_mc (src/drinkme/codec/radix_ops.py:
 * 351-398): x is bf16 or fp32 (`x_dtype`, row stride C), 1 <= M <= 8
 * (DM_EINVAL outside, the ValueError of radix_ops.py:384-385), bias is a
 * bf16 [rows] vector or NULL, out is [M, rows] row-major in `out_dtype`.
 * Column m of an M-row call is bitwise the M=1 call on row m. x may start
 * at any address aligned to its element size (DM_EINVAL otherwise): for a
 * sip tensor, fp32 rows and bf16 rows off a 16-byte boundary are first
 * staged (split or copied) into the tensor's own buffer, with the same
 * result bits. Uses the tensor's own scratch: calls on one tensor must not
 * overlap on the GPU. */
int dm_gemv(const dm_tensor *t, const void *x, int32_t x_dtype, int64_t M, const void *bias, void *out,
            int32_t out_dtype, void *stream, char *err, size_t err_len);

/* dm_gemv for callers that cannot allocate device memory at call time — a
 * serving engine that has given all free HBM to its own pool before decoding
 * starts, or a decode loop that must not call cudaMalloc (which can
 * synchronise the device). No counterpart in the reference. Same arguments,
 * results and errors as dm_gemv (bitwise the same outputs); the only
 * difference is where the kernel's scratch lives: one static array in the
 * library's device memory (about 1.45 MiB, held on every GPU that loads the
 * library until exit) instead of the tensor's own buffers. This call makes no
 * cudaMalloc, cudaFree or other allocating call. Limits of that array
 * (DM_EINVAL beyond them): tensors or row shards of at most 262,144 rows;
 * at most 32,768 columns for activations that are staged in it (fp32, or
 * bf16 off a 16-byte boundary). The first call on a device
 * looks the array's device address up (cudaGetSymbolAddress): make it before
 * capturing a CUDA graph on that device; the address is kept for the life of
 * the process, so the device's primary context must not be reset in between.
 * Every call shares the array, so calls that overlap on the GPU (on any
 * tensor, any stream) race. */
int dm_gemv_noalloc(const dm_tensor *t, const void *x, int32_t x_dtype, int64_t M, const void *bias, void *out,
                    int32_t out_dtype, void *stream, char *err, size_t err_len);

/* The launch schedule of a sip tensor's GEMV — this library's counterpart of
 * the reference's per-tensor launch row (src/drinkme/codec/radix_schedule.py:
 * 187-206 TABLES, 394-417 select; its Triton knobs are blocks per program
 * and warps, these are the sm_100a kernel's own). Fields <= 0 (or -1 where
 * noted) take the measured defaults:
 *   slots     staging slots of the unit ring, 1..6 (0: five, six at M = 1
 *             for tensors of 8 or more block columns; fewer when they do not
 *             fit beside the activations);
 *   split     0: choose by cost, 1: stream-K over units, 2: whole 16-row
 *             tiles per CTA;
 *   skew      stream-K: units fewer than the average that the last CTA to be
 *             dispatched gets, 0..64 (-1: 4);
 *   resident  the most block columns whose activations stay resident in
 *             shared memory for the launch, 0..16 (-1: 16; 0: staged with
 *             every unit).
 * Slots and residency change how data is staged, never a result bit; split
 * and skew change which CTA sums which units, so results move within the
 * fp32-accumulation bound (every sum's order still depends on the tensor and
 * its launch alone). Applies to dm_gemv, dm_gemv_noalloc, dm_gemv_gather and
 * dm_decode; DM_EINVAL outside the ranges. */
typedef struct dm_launch {
    int32_t slots, split, skew, resident;
    int32_t prefetch; /* units past the staged ones whose weights each CTA asks into L2 before it waits for the
                         activations (-1: the default, none; 0: none; at most 32) */
} dm_launch;
int dm_tensor_set_launch(dm_tensor *t, const dm_launch *launch, char *err, size_t err_len);

/* What a GEMV of `M` activation rows of `x_dtype` (fp32 rows count three
 * virtual rows each, at most two rows per launch) would launch: the grid (CTAs),
 * the split (1 stream-K, 2 whole tiles), the staging slots, 1 when the
 * activations stay resident, the dynamic shared memory, and the stream-K
 * weight step (0: an even split). Nothing runs. */
typedef struct dm_launch_plan {
    int32_t grid, split, slots, resident, smem_bytes, skew_step;
} dm_launch_plan;
int dm_gemv_plan(const dm_tensor *t, int64_t M, int32_t x_dtype, dm_launch_plan *plan, char *err, size_t err_len);

/* Prefill: y[M, rows] = x[M, C] @ W^T (+ bias) for a prefill chunk (any M >=
 * 1; the module routes M >= 9 here), W a sip tensor (fast_path): the weights
 * are decoded into shared memory and contracted on the tensor cores
 * (tcgen05.mma, fp32 accumulate in tensor memory), the bias added in fp32 and
 * one rounding to `out_dtype`. Replaces the dense arm's decode + GEMM
 * (src/drinkme/codec/radix_kernel_gpu.py:615-636, swap.py:361-378). x is bf16
 * [M, C], 16-byte aligned; `work` is a device workspace of at least
 * dm_prefill_workspace_bytes(t, M) bytes, 16-byte aligned (the activations
 * re-laid out for the tensor core); out is [M, rows]. */
int64_t dm_prefill_workspace_bytes(const dm_tensor *t, int64_t M);
int dm_prefill(const dm_tensor *t, const void *x, int64_t M, const void *bias, void *out, int32_t out_dtype,
               void *work, int64_t work_bytes, void *stream, char *err, size_t err_len);

/* The output gather of a row-sharded linear over NVLink, fused into its GEMV
 * (the exchange the reference lacks: it has no multi-GPU code; this replaces
 * an all-gather after each shard's dm_gemv). Rank `rank` of `world` holds
 * rows [rank * slot, rank * slot + rows) of the linear (its dm_tensor, made
 * with that row range or as a fused tensor of such ranges). Every rank owns a
 * gathered output buffer [M][world * slot] and `world` flag words for this
 * linear, and maps every other rank's (dm_ipc_open); the arrays below give
 * them in this process's address space, index = rank. `gen` and `done` are
 * this rank's own zero-initialised words for this linear. With `wait_flags`
 * and `wait_gen` (this rank's flag words and launch count of the linear the
 * activations depend on) the kernel first waits, bounded, until every rank
 * has published that linear's output. */
typedef struct dm_gather {
    int32_t world, rank;
    int64_t slot;
    void *peer_out[DM_MAX_RANKS];
    uint32_t *peer_flags[DM_MAX_RANKS];
    uint32_t *gen, *done;
    const uint32_t *wait_flags, *wait_gen;
    uint32_t *abort; /* this rank's word, shared by all its linears: set when a wait gives up; later waits then return at once */
    uint32_t wait_polls; /* the most flag polls of one wait before it gives up (0: 2^23, a few seconds) */
} dm_gather;

/* dm_gemv of this rank's rows, the outputs stored into every rank's
 * gathered buffer at [m][rank * slot + row] (no local `out`), then every
 * rank's flag word `rank` of this linear raised to the new launch count.
 * bf16 activations (16-byte aligned), 1 <= M <= 8, a sip tensor; one kernel
 * launch, no host synchronisation (CUDA-graph capturable). A wait that gave
 * up is reported by dm_tensor_check. Kernels of different ranks wait on one
 * another: run one rank per GPU. */
int dm_gemv_gather(const dm_tensor *t, const void *x, int64_t M, const void *bias, int32_t out_dtype,
                   const dm_gather *g, void *stream, char *err, size_t err_len);

/* A sequence of dm_gemv_gather calls in ONE persistent launch (a chain):
 * the reference runs one module call per linear (src/drinkme/codec/
 * swap.py:426-456) and has no counterpart for the sequence; this is the
 * per-linear route with the launches, and their start and drain, taken out.
 * Link i computes this rank's rows of its tensor from `x` into every rank's
 * gathered buffer (g, as dm_gemv_gather; g.wait_flags / g.wait_gen are not
 * read) and raises its flags to the chain's launch count. With wait = j it
 * first waits, bounded, for link j's flags: this launch's output of link j
 * when j < i, the previous launch's when j >= i (none on the first launch).
 * Same result bits as the per-linear calls. A tensor may serve two links
 * only when the later one waits (directly or through others) on the earlier.
 * A PeerGather's flags serve either one chain or per-linear calls, not both.
 * bf16 activations, 16-byte aligned, 1 <= M <= 8, sip tensors on one device.
 * dm_chain_create copies the links' kernel arguments to the device (one
 * allocation; the chain's launch count starts at zero); dm_chain_run is one
 * cooperative kernel launch, no host synchronisation (CUDA-graph
 * capturable); every rank runs its chain the same number of times. */
typedef struct dm_chain dm_chain;
typedef struct dm_chain_link {
    const dm_tensor *t;
    const void *x;    /* bf16 [M][C] */
    const void *bias; /* bf16 [rows] or NULL */
    dm_gather g;
    int32_t wait;     /* -1: none */
} dm_chain_link;
int dm_chain_create(const dm_chain_link *links, int32_t n, int64_t M, int32_t out_dtype, dm_chain **out, char *err,
                    size_t err_len);
int dm_chain_run(const dm_chain *c, void *stream, char *err, size_t err_len);
int dm_chain_destroy(dm_chain *c, char *err, size_t err_len);

/* CUDA IPC of a device allocation (plain peer mappings; no multicast):
 * the 64-byte handle of `dptr` (the start of a cudaMalloc block), and the
 * mapping of a peer's handle on `device` (closed by dm_ipc_close). */
int dm_ipc_handle(const void *dptr, uint8_t *out64, char *err, size_t err_len);
int dm_ipc_open(const uint8_t *handle64, int32_t device, void **dptr, char *err, size_t err_len);
int dm_ipc_close(void *dptr, char *err, size_t err_len);

/* Device memory for gather buffers and flags: cudaMalloc'd and zeroed (the
 * start of the block is what dm_ipc_handle exports). */
int dm_device_alloc(int32_t device, size_t bytes, void **dptr, char *err, size_t err_len);
int dm_device_free(void *dptr, char *err, size_t err_len);

/* The shard's decoded bf16 bit patterns, uint16 [rows, C] — replaces
 * radix_ops.decode_bits (src/drinkme/codec/radix_ops.py:418-427). For a
 * sip tensor (fast_path) `out` must be 16-byte aligned. */
int dm_decode(const dm_tensor *t, uint16_t *out, void *stream, char *err, size_t err_len);

/* The gulp schedule over the ORIGINAL pack layout on the device: one
 * uint16 per block whose byte (k-1) is the word length of nonterminal tier
 * k's stream — replaces radix_ops.prepare_schedule
 * (src/drinkme/codec/radix_ops.py:341-348). Words at or past `nwords` read
 * as zero. */
int dm_prepare_schedule(const uint32_t *data, size_t nwords, const uint32_t *offsets, int64_t C,
                        const int32_t *host_widths, int32_t nwidths, int32_t block_size, int64_t nblocks,
                        uint16_t *out, void *stream, char *err, size_t err_len);

/* y[M, R] = x[M, C] @ w[R, C]^T (+ bias) over a raw row-major bf16 weight
 * — replaces radix_ops.gemv_narrow (src/drinkme/codec/radix_ops.py:
 * 401-415) and serves the raw lm_head (swap.stock_linear, swap.py:
 * 681-707). 1 <= M <= 8; fp32 accumulate, bias in fp32, one rounding. w
 * and x at any address aligned to their element size: 16-byte loads when
 * both are 16-byte aligned and C % 8 == 0, a scalar loop otherwise. */
int dm_gemv_raw(const void *w, int64_t R, int64_t C, const void *x, int32_t x_dtype, int64_t M,
                const void *bias, void *out, int32_t out_dtype, void *stream, char *err, size_t err_len);

/* The pack encoder (src/drinkme/codec/radix_native.cpp:57-166 `plan` +
 * `encode`; radix.py:77-136 for any block size): uint16 [R, C] bf16 bits
 * -> the pack arrays, byte-identical to the reference's. Two calls:
 * dm_pack_plan fills host_palette (covered entries) and host_offsets
 * (R*NB+1) and returns the payload word count in *nwords; dm_pack_encode
 * then writes host_data[nwords]. `threads` <= 0 uses every host core. */
int dm_pack_plan(const uint16_t *host_bits, int64_t R, int64_t C, const int32_t *host_widths, int32_t nwidths,
                 int32_t block_size, int32_t threads, uint8_t *host_palette, uint32_t *host_offsets,
                 uint64_t *nwords, char *err, size_t err_len);
int dm_pack_encode(const uint16_t *host_bits, int64_t R, int64_t C, const int32_t *host_widths,
                   int32_t nwidths, int32_t block_size, int32_t threads, const uint8_t *host_palette,
                   const uint32_t *host_offsets, uint32_t *host_data, uint64_t nwords, char *err, size_t err_len);

/* Decodes a pack as stored — its word stream and block directory copied to
 * the device unchanged (d_data: nwords words, d_offsets: R*NB+1 entries),
 * no device layout — to bf16 bit patterns d_out [R][C] (radix.py:241-278,
 * radix_native.cpp:168-209). The host copies of the palette and directory
 * are validated first (radix.py:174-238). A warp per block; for
 * verification and for packs held in device memory as they are. */
int dm_decode_pack(const uint8_t *host_palette, size_t npalette, const uint32_t *host_offsets, size_t noffsets,
                   size_t nwords, int64_t R, int64_t C, const int32_t *host_widths, int32_t nwidths,
                   int32_t block_size, const uint32_t *d_data, const uint32_t *d_offsets, uint16_t *d_out,
                   void *stream, char *err, size_t err_len);

/* The same encoder on the GPU (radix_native.cpp:57-166 `plan` / `encode`,
 * the writers behind radix.py:77-136 `pack_array`), for bits already in
 * device memory: dm_pack_plan_device histograms the exponents and counts
 * every block's words on the device and fills host_palette, host_offsets
 * (R*NB+1) and *nwords on the host (it synchronises `stream`);
 * dm_pack_encode_device then writes the nwords payload words into d_data
 * (device memory of the bits' GPU), byte-identical to dm_pack_encode, and
 * synchronises `stream`. Temporary device memory comes from the stream-
 * ordered allocator. */
int dm_pack_plan_device(const uint16_t *d_bits, int64_t R, int64_t C, const int32_t *host_widths, int32_t nwidths,
                        int32_t block_size, uint8_t *host_palette, uint32_t *host_offsets, uint64_t *nwords,
                        void *stream, char *err, size_t err_len);
int dm_pack_encode_device(const uint16_t *d_bits, int64_t R, int64_t C, const int32_t *host_widths,
                          int32_t nwidths, int32_t block_size, const uint8_t *host_palette,
                          const uint32_t *host_offsets, uint32_t *d_data, uint64_t nwords, void *stream, char *err,
                          size_t err_len);

/* The fused operations around the packed Linears in a batch-1 decode step
 * (no counterpart in the reference's path: it runs transformers' own
 * modules there, src/drinkme/serving/cudagraph.py). bf16 storage, fp32
 * arithmetic; positions are read from device memory, so one captured graph
 * serves every step.
 *   dm_step_add_rmsnorm: h += delta (when delta is not null, rounded to
 *     bf16), out = bf16(h * rsqrt(mean(h^2) + eps)) * w, over n values.
 *   dm_step_qk_rope_cache: per head of the fused q|k|v row, RMSNorm of q and
 *     k heads (weights qn, kn), the rotary embedding at *pos (cos/sin tables
 *     [max_len][head_dim / 2] fp32), q into q_out, k and v into row *pos of
 *     the layer's caches [max_len][nkv][head_dim]. head_dim 128.
 *   dm_step_attention: grouped-query attention of q [nh][head_dim] over the
 *     cache rows 0..*pos into out [nh][head_dim]; `work` holds
 *     dm_step_attention_workspace_bytes(nh, head_dim, max_len) bytes.
 *   dm_step_silu_mul: out[i] = silu(gu[i]) * gu[n + i]. */
int dm_step_add_rmsnorm(void *h, const void *delta, const void *w, void *out, int64_t n, float eps, void *stream,
                        char *err, size_t err_len);
int dm_step_qk_rope_cache(const void *qkv, const void *qn, const void *kn, const float *cos_table,
                          const float *sin_table, const int64_t *pos, void *q_out, void *kcache, void *vcache,
                          int32_t nh, int32_t nkv, int32_t head_dim, float eps, void *stream, char *err,
                          size_t err_len);
int64_t dm_step_attention_workspace_bytes(int32_t nh, int32_t head_dim, int64_t max_len);
int dm_step_attention(const void *q, const void *kcache, const void *vcache, const int64_t *pos, int64_t max_len,
                      void *out, float *work, int32_t nh, int32_t nkv, int32_t head_dim, void *stream, char *err,
                      size_t err_len);
int dm_step_silu_mul(const void *gu, void *out, int64_t n, void *stream, char *err, size_t err_len);
/* dm_step_qk_rope_cache and dm_step_attention in one launch: the q/k norms,
 * rotary and cache write of row *pos, the split attention and its combine
 * (the last CTA of each kv head combines, then resets its counter). `work`
 * holds dm_step_attention_block_workspace_bytes bytes, zeroed before the
 * first call. Same result bits as the two entry points. */
int64_t dm_step_attention_block_workspace_bytes(int32_t nh, int32_t nkv, int32_t head_dim, int64_t max_len);
int dm_step_attention_block(const void *qkv, const void *qn, const void *kn, const float *cos_table,
                            const float *sin_table, const int64_t *pos, void *kcache, void *vcache, int64_t max_len,
                            void *out, void *work, int32_t nh, int32_t nkv, int32_t head_dim, float eps, void *stream,
                            char *err, size_t err_len);

/* Reads and clears the tensor's device error word (a kernel's bounded
 * wait that gave up writes it). Synchronises the tensor's device. */
int dm_tensor_check(const dm_tensor *t, int32_t *device_error, char *err, size_t err_len);

#ifdef __cplusplus
}
#endif

#endif /* DRINKME_B200_H */
