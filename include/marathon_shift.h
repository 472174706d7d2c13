/*
 * marathon_shift.h — C ABI of the B200 position-shifted KV reuse path.
 *
 * Every entry point takes plain device pointers, element strides and a CUDA
 * stream (passed as void* so the header needs no CUDA include), writes its
 * results in place into caller-owned memory, allocates nothing, and returns a
 * status code (MSHIFT_OK on success).  Launches are asynchronous on `stream`.
 *
 * Two errors are reported differently:
 *   - argument errors found on the host (null pointer, unsupported dtype or
 *     head geometry, bad sizes) return MSHIFT_EINVAL / MSHIFT_EUNSUPPORTED and
 *     launch nothing;
 *   - per-token errors only the device can see (a slot outside the paged
 *     cache, a store position outside the session buffer, a bad session or
 *     table index inside a run descriptor) skip that token and OR an
 *     MSHIFT_EBIT_* bit into *err, which the caller zeroes beforehand and reads
 *     after the stream has synchronised.  No kernel traps or faults on a bad
 *     descriptor.  While a batched load or save runs, bits 8..31 of *err
 *     count the tiles its CTAs have claimed (they are cleared again before the
 *     launch completes), so one status word must not be shared by launches
 *     that can run at the same time; launches ordered on one stream may share
 *     it and accumulate their flags.  A CTA's claims strictly increase within
 *     a launch; a CTA that draws one that does not (the counter was reset by
 *     another launch on the same word) sets MSHIFT_EBIT_CLAIM and stops.
 *
 * Layout vocabulary (shared with the Python package marathon_b200):
 *   store    one buffer per (session, layer): [capacity, heads, 2*head_size],
 *            row index = absolute token position, K in [..., :head_size],
 *            V in [..., head_size:].  Strides st_tok / st_head in elements.
 *   paged    vLLM's paged KV cache for one layer.  A token's K row for head h
 *            lives at k_base + blk*blk_stride + off*off_stride + h*head_stride
 *            and its V row at the same offset from v_base, where
 *            blk = slot / block_size, off = slot % block_size.  This covers
 *            the fused NHD / HND layouts (v_base = k_base + head_size) and the
 *            split (2, blocks, block_size, heads, head_size) layouts alike.
 *   run      a contiguous run of tokens: store positions
 *            [store_start, store_start + len) paired with paged slots that are
 *            either listed explicitly (slots[len]) or derived from a block
 *            table: slot(t) = block_table[(paged_start+t)/bs]*bs + (paged_start+t)%bs.
 *   table    rotation table of one delta: float[2][half], cos then sin of
 *            fp32(delta) * inv_freq[i], i < half = rotary/2.
 */
#ifndef MARATHON_SHIFT_H
#define MARATHON_SHIFT_H

#include <stdint.h>

#if defined(__GNUC__)
#define MSHIFT_API __attribute__((visibility("default")))
#else
#define MSHIFT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define MSHIFT_OK 0
#define MSHIFT_EINVAL 1       /* bad argument (null pointer, size, stride)  */
#define MSHIFT_EUNSUPPORTED 2 /* dtype / head_size / rotary not compiled    */
#define MSHIFT_ECUDA 3        /* a CUDA runtime call failed                 */
#define MSHIFT_ETOOBIG 4      /* exceeds the static scratch of mshift_load_noalloc */

/* ---- device error bits ORed into *err ---------------------------------- */
#define MSHIFT_EBIT_SLOT 1u    /* slot < 0 or slot >= num_blocks*block_size  */
#define MSHIFT_EBIT_STORE 2u   /* store position < 0 or >= session capacity  */
#define MSHIFT_EBIT_SESSION 4u /* run.session outside [0, n_sessions) or null buffer */
#define MSHIFT_EBIT_TABLE 8u   /* run.table outside [-1, n_tables)           */
#define MSHIFT_EBIT_TIMEOUT 16u /* a bulk copy did not complete in time; the launch stopped */
#define MSHIFT_EBIT_CLAIM 32u   /* the tile-claim counter went backwards (the status word
                                   was shared with a launch in flight); the launch stopped */

/* ---- element types ----------------------------------------------------- */
#define MSHIFT_BF16 0
#define MSHIFT_F16 1
#define MSHIFT_F32 2
#define MSHIFT_E4M3 3 /* float8_e4m3fn codes, per-layer scale */

/* Geometry of one layer's paged cache (identical for every layer). */
typedef struct mshift_paged {
    int64_t blk_stride;  /* elements between consecutive blocks            */
    int64_t off_stride;  /* elements between consecutive in-block offsets  */
    int64_t head_stride; /* elements between consecutive heads             */
    int64_t num_blocks;  /* blocks in the cache, for the slot bounds check */
    int32_t block_size;
    int32_t heads;      /* KV heads held by this rank                      */
    int32_t head_size;  /* D: K row and V row are D elements each          */
    int32_t dtype;      /* MSHIFT_BF16 / F16 / F32 / E4M3                  */
} mshift_paged;

/* One run of tokens moved between a session's store and the paged cache. */
typedef struct mshift_run {
    int64_t store_start;        /* store position of the run's first token          */
    int64_t paged_start;        /* logical position of the first token (block-table mode) */
    const int64_t* slots;       /* device [len] flat slots, or NULL for block-table mode */
    const int32_t* block_table; /* device block table of the request (block-table mode) */
    int32_t block_table_len;    /* entries in block_table (bounds check)            */
    int32_t len;                /* tokens in the run (> 0)                          */
    int32_t session;            /* row of store_ptrs / store_caps                   */
    int32_t table;              /* load: rotation table row, -1 = copy K unrotated   */
    int32_t tile_begin;         /* sum over earlier runs of ceil(len/tile_tokens)   */
    int32_t reserved;           /* zero                                             */
} mshift_run;                   /* 56 bytes, 8-byte aligned                         */

/*
 * Rotation tables for n deltas: tables[d][0][i] = cosf(a), tables[d][1][i] =
 * sinf(a) with a = fp32(deltas[d]) * inv_freq[i] rounded to fp32 -- the
 * values torch's fp32 cos / sin give on a CUDA device, i.e. the reference's
 * own tables as its GPU path builds them.  One launch for all deltas.
 * Replaces: marathon rope_shift (src/marathon/shift_kernels.py:68-84), whose
 * cos/sgn/partner tables are this table plus a sign flip and a permutation.
 */
MSHIFT_API int mshift_rope_tables(const int64_t* deltas, int32_t n, const float* inv_freq,
                       int32_t half, float* tables, void* stream);

/*
 * One layer, one run: write src rows [n, heads, 2*head_size] into the paged
 * cache at slots[n], K rotated by `table` (NULL = plain scatter).  V is always
 * copied bit for bit.  E4M3 (dequantise -> rotate -> requantise with the
 * layer's K scale): the scale cancels, so the codes' values are rotated in
 * fp32 and rounded once to e4m3 (saturating, nearest even) -- within one
 * e4m3 step of the step-by-step result.  k_scale (device, the layer's K
 * scale) is therefore not read and may be NULL.
 * Replaces: the Triton launch _shift_scatter_kernel[grid](...) of
 * scatter_shifted (src/marathon/shift_kernels.py:89-132, :166-210).
 */
MSHIFT_API int mshift_scatter_shifted(const void* src, int64_t src_tok_stride,
                           int64_t src_head_stride, int64_t n, void* k_base,
                           void* v_base, const mshift_paged* paged,
                           const int64_t* slots, const float* table,
                           int32_t rotary, const float* k_scale, uint32_t* err,
                           void* stream);

/*
 * Batched load: every run x every layer in one persistent launch.  For layer
 * l and run r, store_ptrs[r.session * n_layers + l] rows
 * [r.store_start, +r.len) are written to the paged cache of layer l
 * (k_ptrs[l], v_ptrs[l]) with K rotated by tables[r.table].  E4M3 caches are
 * rotated as in mshift_scatter_shifted; k_scales (per-layer K scales) is not
 * read and may be NULL.
 * tiles_per_layer = sum over runs of ceil(len / tile_tokens); each run's
 * tile_begin is the exclusive prefix of that sum (mshift_plan_tiles fills it).
 * tile_tokens is 1..512 (else MSHIFT_EINVAL); mshift_save takes the same.
 * With n_tables > 0 the kernel is launched with programmatic stream
 * serialization: its CTAs may start while the kernel just before it in the
 * stream (normally mshift_rope_tables) finishes, and wait for that kernel's
 * completion before touching memory, so stream order holds as usual.
 * Replaces: the per-layer loop of MarathonShiftConnector.start_load_kv
 * (src/marathon/vllm_shift_connector.py:495-518) = ShiftStore.read
 * (src/marathon/shift_store.py:238-250) + scatter_shifted per layer and load.
 */
MSHIFT_API int mshift_load(const mshift_paged* paged, int32_t rotary, const mshift_run* runs,
                int32_t n_runs, int32_t tile_tokens, int32_t tiles_per_layer,
                int32_t n_layers, void* const* store_ptrs, const int64_t* store_caps,
                int32_t n_sessions, int64_t st_tok, int64_t st_head,
                void* const* k_ptrs, void* const* v_ptrs, const float* tables,
                int32_t n_tables, const float* k_scales, uint32_t* err, void* stream);

/*
 * Batched save: the mirror of mshift_load without rotation.  For layer l and
 * run r, the paged rows of the run's slots are copied bit for bit into
 * store_ptrs[r.session * n_layers + l] rows [r.store_start, +r.len).
 * Replaces: MarathonShiftConnector._gather + ShiftStore.write per layer
 * (src/marathon/vllm_shift_connector.py:418-442, :539-553;
 * src/marathon/shift_store.py:225-236).
 */
MSHIFT_API int mshift_save(const mshift_paged* paged, const mshift_run* runs, int32_t n_runs,
                int32_t tile_tokens, int32_t tiles_per_layer, int32_t n_layers,
                void* const* store_ptrs, const int64_t* store_caps,
                int32_t n_sessions, int64_t st_tok, int64_t st_head,
                void* const* k_ptrs, void* const* v_ptrs, uint32_t* err,
                void* stream);

/*
 * Host helper: fill runs[i].tile_begin (host array) and return
 * tiles_per_layer, or -1 if a run has len <= 0 or the sum overflows int32.
 * Replaces nothing in the reference (its loop launched one kernel per layer).
 */
MSHIFT_API int32_t mshift_plan_tiles(mshift_run* runs, int32_t n_runs, int32_t tile_tokens);

/* Tile size the library would pick for `heads` heads (tokens per tile). */
MSHIFT_API int32_t mshift_default_tile_tokens(int32_t heads);

/*
 * Load kernel selection, process-wide.  MSHIFT_KERNEL_LSU: every byte through
 * 128-bit loads/stores.  MSHIFT_KERNEL_BULK: each tile's store rows reach
 * shared memory in one TMA bulk copy (cp.async.bulk, mbarrier ring, producer
 * warp) when the store rows are dense; otherwise the LSU kernel runs.
 * MSHIFT_KERNEL_AUTO (default): BULK for e4m3 caches, LSU for the others (the
 * faster of the two for each on B200).  Returns the previous kind, or -1 for
 * an unknown kind.  No counterpart in the reference (its one Triton kernel had
 * no alternative).
 */
#define MSHIFT_KERNEL_LSU 0
#define MSHIFT_KERNEL_BULK 1
#define MSHIFT_KERNEL_AUTO 2
MSHIFT_API int mshift_set_load_kernel(int kind);

/*
 * Diagnostic hook for the TMA load kernel's timeout path, process-wide.
 * rounds >= 0 bounds the first full-barrier wait of every consumer warp of
 * every later TMA load launch to that many try_wait rounds (0: it gives up at
 * once), so a test can make that wait run out on purpose: the launch then
 * sets MSHIFT_EBIT_TIMEOUT, writes nothing more, waits (with the normal bound)
 * for the bulk copies it already issued, and returns.  rounds < 0 restores the
 * normal bound.  Returns the previous setting (-1 = normal).  No counterpart in
 * the reference (its Triton kernel had no waits).
 */
MSHIFT_API int32_t mshift_debug_first_wait(int32_t rounds);

/* 1 if (dtype, head_size, rotary) has a compiled kernel, else 0. */
MSHIFT_API int mshift_supported(int32_t dtype, int32_t head_size, int32_t rotary);

/* Version string and the text of a status code. */
MSHIFT_API const char* mshift_version(void);
MSHIFT_API const char* mshift_strerror(int status);

/* Last CUDA error text seen by the library on this thread (for MSHIFT_ECUDA). */
MSHIFT_API const char* mshift_last_cuda_error(void);

/*
 * Allocation-free batched load.  No counterpart in the reference: it exists
 * for callers that cannot allocate device memory at load time -- a server
 * whose whole device pool is handed out at start-up, or a host binding that
 * can only pass pointers it already owns.  Same work and arguments as
 * mshift_rope_tables + mshift_load, except that the caller passes the deltas
 * (device int64[n_deltas]) and inv_freq (device float[rotary/2]) instead of a
 * table buffer: the tables are built in a fixed 256 KiB array inside the
 * library's device image (run r's `table` indexes `deltas`).  Limits: at most
 * mshift_noalloc_max_deltas() (256) deltas and rotary <= 256; beyond that the
 * call returns MSHIFT_ETOOBIG and launches nothing.  The array is shared by
 * all calls: calls whose work overlaps on the GPU race on it.  The first call
 * on a device resolves the array's address (cudaGetSymbolAddress) with that
 * device current; make that first call before any stream capture.
 */
MSHIFT_API int mshift_load_noalloc(const mshift_paged* paged, int32_t rotary,
                const mshift_run* runs, int32_t n_runs, int32_t tile_tokens,
                int32_t tiles_per_layer, int32_t n_layers, void* const* store_ptrs,
                const int64_t* store_caps, int32_t n_sessions, int64_t st_tok,
                int64_t st_head, void* const* k_ptrs, void* const* v_ptrs,
                const int64_t* deltas, int32_t n_deltas, const float* inv_freq,
                const float* k_scales, uint32_t* err, void* stream);

/* Most distinct deltas one mshift_load_noalloc call accepts. */
MSHIFT_API int32_t mshift_noalloc_max_deltas(void);

/*
 * Store tier off the GPU: staged copies.  A store whose buffers live in
 * pinned host memory or on another GPU is never read by a kernel; its rows
 * are copied (copy engines, one cudaMemcpyAsync per range, in array order,
 * cudaMemcpyDefault) into a device staging buffer that mshift_load reads, and
 * mshift_save's staging rows are copied back the same way.  `copies` is a
 * host array; ranges of zero bytes are skipped.  Host ranges must be pinned
 * for the copy to be asynchronous.  No counterpart in the reference: its
 * store is device-only (docs/protocol.md:49, src/marathon/shift_store.py:251-253).
 */
typedef struct mshift_copy {
  void* dst;
  const void* src;
  int64_t bytes;
} mshift_copy;

MSHIFT_API int mshift_stage(const mshift_copy* copies, int32_t n, void* stream);

/*
 * Enable direct (NVLink) copies from `peer_device` to the current device, for
 * a store tier on another GPU.  MSHIFT_OK if enabled or already enabled,
 * MSHIFT_EUNSUPPORTED if the pair has no peer access.  Kernels never
 * dereference peer memory: only mshift_stage copies read it.
 */
MSHIFT_API int mshift_enable_peer(int32_t peer_device);

#ifdef __cplusplus
}
#endif

#endif /* MARATHON_SHIFT_H */
