/*
 * hawk_b200.h -- the C ABI of the B200 (sm_100a) execution path for hawk kernels.
 *
 * The reference runs a built kernel through its native binding hawk._core
 * (src/hawk_core.cpp, a nanobind module): it loads the artifact, self-checks
 * its ABI exports, packs every plane into a by-value mirror in an argument
 * block and calls the entry over a partition [base, base + count) of nSamples.
 * This library is the device twin of that binding, with plain C types only:
 * each entry point below names the hawk._core member it replaces.  Beyond it,
 * the library finishes sample-sum rows into cells on the device (the
 * reference does that in numpy, hawk/_cells.py:94-119).
 *
 * Conventions.
 *   - Every function returns HKB_OK (0) or a nonzero status; the message of
 *     the last failure on the calling thread is hkb_last_error().
 *   - Pointers to planes are device pointers (CUDA unified addressing);
 *     `stream` is a cudaStream_t (NULL: the legacy default stream).  Launch
 *     entry points are asynchronous on that stream and allocate nothing.
 *   - A library handle is usable from any thread; an argument block is not
 *     synchronised -- one block per thread, or the caller orders the calls
 *     (the reference's HostKernel lock, hawk/runtime.py:46-54).
 */
#ifndef HAWK_B200_H
#define HAWK_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */
#define HKB_OK 0
#define HKB_ERR_ARGUMENT 1   /* a bad argument (slot out of range, null pointer, unknown kind) */
#define HKB_ERR_CUDA 2       /* a CUDA runtime call failed (message names it) */
#define HKB_ERR_ABI 3        /* an artifact whose self-check exports disagree */
#define HKB_ERR_NOT_FOUND 4  /* no such entry in the artifact */
#define HKB_ERR_RANGE 5      /* a partition or size outside what the call accepts */

/* Sample-sum ops (hawk/emit/wrapper.py:719 SAMPLE_SUM_OP_CODE) and element types. */
#define HKB_OP_SUM 0
#define HKB_OP_MAX 1
#define HKB_OP_MIN 2
#define HKB_F64 0
#define HKB_F32 1

/* Rows per leaf of the ordered finish tree (hawk/_cells.py:25-27: 256 slots x 16 terms). */
#define HKB_LEAF_ROWS 4096

typedef struct hkb_library hkb_library;   /* one loaded sm_100a artifact (CUBIN) */
typedef struct hkb_entry hkb_entry;       /* one __global__ entry of it */
typedef struct hkb_argblock hkb_argblock; /* the by-value argument cells of an entry */

/* The message of the last failed call on this thread ("" if none). */
const char* hkb_last_error(void);

/* ----------------------------------------------------------- build facts */

/* hawk._core.build_digest() (src/hawk_core.cpp:523-530): the sha256 of the
 * sources this library was built from. */
const char* hkb_build_digest(void);

/* hawk._core.layout_sizes() (src/hawk_core.cpp:531-537): sizeof GRefMirror,
 * ScalarHandle, IntHandle, the index type and PartitionTriple -- 40, 32, 32, 8, 24. */
int hkb_layout_sizes(uint64_t out[5]);

/* The number of CUDA devices this process sees (0 without a driver). */
int hkb_device_count(int* count);

/* -------------------------------------------------------------- library */

/* hawk._core.HostLibrary(path) (src/hawk_core.cpp:354-427, :654-662): load an sm_100a
 * CUBIN image onto `device` and check its exports eagle_abi_tag ==
 * "aether-abi/2" and eagle_layout_sizes == hkb_layout_sizes; a mismatch is
 * HKB_ERR_ABI naming the field. */
int hkb_library_load(const void* image, size_t size, int device, hkb_library** out);
int hkb_library_load_file(const char* path, int device, hkb_library** out);
void hkb_library_free(hkb_library* lib);

/* The unit's error word (0 when every bounded wait of its entries completed;
 * bit 1: a staged tile did not arrive in time, 2: a stage was not released in
 * time, 4: copies were still in flight when a CTA gave up), read after the
 * launches it covers have completed; `clear` resets it.  A unit without the
 * word reads 0.  The reference's host target has no device waits to report. */
int hkb_library_errors(hkb_library* lib, unsigned* flags, int clear);

/* HostLibrary.entry(name) (src/hawk_core.cpp:663-667): the entry `name`.  A
 * team entry (a stage of team-form linear algebra, hawk/ir/team.py) exports
 * its threads per block as hk_team_threads__<name> and launches one block per
 * lane; an entry's dynamic shared memory is hk_dynamic_smem_bytes__<name>,
 * else the unit's hk_dynamic_smem_bytes. */
int hkb_library_entry(hkb_library* lib, const char* name, hkb_entry** out);

/* Facts of an entry: registers per thread, resident blocks per SM at its
 * block size, the block size, and the grid a launch of `count` samples takes. */
int hkb_entry_info(hkb_entry* entry, int* regs, int* blocks_per_sm, int* block, int64_t count,
                   int64_t* grid);

/* --------------------------------------------------------- argument block */

/* hawk._core.ArgBlock(descriptor) (src/hawk_core.cpp:185-226, :598-604): one cell per
 * slot, in arg_spec order; kinds are "gref", "handle", "int_handle", "f64",
 * "f32", "int", "nsamples" (hawk/runtime.py:96-118). */
int hkb_argblock_create(const char* const* kinds, size_t n, hkb_argblock** out);
void hkb_argblock_free(hkb_argblock* block);

/* ArgBlock.bind(slot, ptr, samples, stride, device_type, device_id)
 * (src/hawk_core.cpp:228-273, :605-613): a plane slot takes the device pointer and the
 * plane's sample extent (a GRef plane's component pitch is samples * stride);
 * a by-value slot copies the value at host address `ptr`. */
int hkb_argblock_bind(hkb_argblock* block, size_t slot, uintptr_t ptr, uint64_t samples,
                      uint64_t stride, int32_t device_type, int32_t device_id);

/* ArgBlock.rebind(slots, ptrs) (src/hawk_core.cpp:275-305, :614-630): swap the data
 * pointers of plane slots in one call; a by-value slot is refused. */
int hkb_argblock_rebind(hkb_argblock* block, const int64_t* slots, const int64_t* ptrs, size_t n);

/* ------------------------------------------------------------------ launch */

/* HostEntry.run(block, base, count, nSamples) (src/hawk_core.cpp:431-442, :642-653):
 * run the entry over samples [base, base + count) of nSamples on `stream`
 * (asynchronous).  A kernel with sample sums needs base % 32 == 0.  A team
 * entry runs lanes [base, base + count), each by one block of its team.  A
 * team stage over keys, lane chunks or target cells (it exports
 * hk_team_spans_run__<entry> = 1; hawk/_lane_bind.py:123-134) takes base 0
 * and count = its teams, which nSamples does not bound; the caller sizes its
 * scratch planes for those teams as hawk/_lane_bind.py:137-145 does. */
int hkb_entry_launch(hkb_entry* entry, hkb_argblock* block, int64_t base, int64_t count,
                     int64_t n_samples, void* stream);

/* The persistent entry of an automatic stepping kernel, `<kernel>_persist`
 * (the reference emits it in hawk/emit/cuda.py:464-707; its runner lives in the
 * absent eagle package): a resident grid whose lanes claim samples of
 * [base, base + count) off `*next` (a uint32 the caller zeroes), run each to
 * its finish or the `fused_steps` budget, write it back and claim the next.
 * `util` (two uint64: steps run, lane slots offered), `steps` (uint32, maxed
 * with the longest per-sample trip count) and `stepsum` (uint64) may be null;
 * `chunk` is the trips between claims (0: whole samples); `grid` the blocks
 * (0: every resident slot the entry's occupancy allows, capped by count).
 * count must be below 2^31. */
int hkb_entry_launch_persist(hkb_entry* entry, hkb_argblock* block, int64_t base, int64_t count,
                             int64_t n_samples, uint32_t* next, uint64_t* util, uint32_t* steps,
                             uint64_t* stepsum, uint32_t chunk, int64_t grid, void* stream);

/* The contiguous-range entry of an automatic stepping kernel, `<kernel>_range`
 * (the reference emits it in hawk/emit/cuda.py:709-784; its runner lives in
 * the absent eagle package): every sample of [base, base + count) on one lane
 * of a grid-stride frame, the fused_steps word 1 running the single step, any
 * other word the fused body's head, trips and tail -- the bits of one launch
 * of the kernel's own entry with that word.  `steps` (uint32, maxed with each
 * sample's steps this launch) and `stepsum` (uint64, their sum) may be null;
 * the caller zeroes them.  Samples finished on entry count into the finished
 * counter with those finishing in the launch. */
int hkb_entry_launch_range(hkb_entry* entry, hkb_argblock* block, int64_t base, int64_t count,
                           int64_t n_samples, uint32_t* steps, uint64_t* stepsum, void* stream);

/* ---------------------------------------------- cells: the ordered finish */

/* The device form of hawk/_cells.py:finish for `ncols` columns (<= 8) of
 * `rows` rows each: stage one writes one (hi, comp) partial per leaf of
 * HKB_LEAF_ROWS rows, stage two folds the leaves pairwise and writes the cell.
 * hi[k] / comp[k] are device pointers to column k's rows (comp may be NULL for
 * max/min); dtype is HKB_F64 or HKB_F32; op is an HKB_OP_*.
 *
 * hkb_cells_leaves: leaf_hi / leaf_comp hold ncols * ceil(rows / 4096) values
 *   (column k at k * leaves).
 * hkb_cells_tree: reads ncols * leaves partials from leaf_hi / leaf_comp
 *   (overwritten), writes out[k] = the cell of column k.
 * hkb_cells_finish: both; `scratch` holds hkb_cells_scratch_bytes(...) bytes. */
int hkb_cells_leaves(int op, int dtype, int ncols, const void* const* hi, const void* const* comp,
                     int64_t rows, void* leaf_hi, void* leaf_comp, void* stream);
int hkb_cells_tree(int op, int dtype, int ncols, void* leaf_hi, void* leaf_comp, int64_t leaves,
                   void* out, void* stream);

/* The same pairwise levels over `count` partials per column, leaf j of column k
 * at element [k * col_stride + j * elem_stride] of hi / comp (in place).  With
 * out_comp non-null the root's (hi, comp) pair of each column is written to
 * out[k] / out_comp[k] instead of hi + comp: the root of an aligned subtree of
 * a larger tree (every rank holding the same power-of-two leaf count is one),
 * which a later call over the subtree roots finishes bit-identically to one
 * tree over all leaves (no counterpart in the reference: its finish is one
 * host tree, hawk/_cells.py:94-119). */
int hkb_cells_tree_ex(int op, int dtype, int ncols, void* hi, void* comp, int64_t count, int64_t elem_stride,
                      int64_t col_stride, void* out, void* out_comp, void* stream);
size_t hkb_cells_scratch_bytes(int dtype, int ncols, int64_t rows);
int hkb_cells_finish(int op, int dtype, int ncols, const void* const* hi, const void* const* comp,
                     int64_t rows, void* scratch, void* out, void* stream);

/* ---------------------------------------------- cells without allocation */

/* No counterpart in the reference: hkb_cells_finish for callers that cannot
 * allocate device memory when they finish a reduction (a host framework that
 * owns every device allocation and gives its plugins only their inputs and
 * outputs; a loop whose memory budget is fixed before it starts).  The leaf
 * partials live in a static device array of the library, 2 x
 * HKB_NOALLOC_LEAF_CAP doubles (128 KiB), which every GPU that loads the
 * library holds until the process exits; the call allocates nothing.
 *
 * Limit: ncols * ceil(rows / 4096) <= HKB_NOALLOC_LEAF_CAP, else HKB_ERR_RANGE
 * (8192 leaves: 33.5M rows for one column).  The first call on a device looks
 * up the array's device address (cudaGetSymbolAddress) and caches it; make
 * that first call before capturing any stream.  The cached address belongs to
 * the device's primary context: after cudaDeviceReset on a device, reload the
 * library in a new process before calling this again.  All calls share the one array:
 * calls that can overlap on the GPU (different streams, different host threads)
 * race on it and must be ordered by the caller.  Every partial is written
 * before it is read within a call, so no state carries between calls. */
#define HKB_NOALLOC_LEAF_CAP 8192
int hkb_cells_finish_noalloc(int op, int dtype, int ncols, const void* const* hi, const void* const* comp,
                             int64_t rows, void* out, void* stream);

/* ------------------------------------- cells across GPUs over peer memory */

/* The last step of a sharded finish in one launch over NVLink, replacing an
 * NCCL all-gather of the ranks' subtree roots (no counterpart in the
 * reference: its ranks finish on the host, tests/mpi/test_hawk_rank_oracle.py:
 * 94-168).  Each rank holds the same power-of-two number of leaves of every
 * column (an aligned subtree of the one-device tree, as for
 * hkb_cells_tree_ex).  One rank's exchange area lives in its own device
 * memory: for each of two round parities, every rank's (hi, comp) root of
 * every column, each 32-bit half of a value in an 8-byte word beside the
 * round's tag.  hkb_peer_finish folds this rank's leaves to its root (the
 * pairwise levels of hkb_cells_tree), stores the root's tagged words into
 * every rank's area with plain peer stores, waits until every rank's words of
 * this round carry the tag in its own area, and runs the last pairwise levels
 * over the ranks' roots in rank order: the same tree, bit for bit, as one
 * hkb_cells_tree over all ranks' leaves.
 *
 * leaf_hi / leaf_comp hold this rank's `leaves` partials of each of the area's
 * ncols columns, column by column (ncols x leaves), and are folded in place;
 * out receives ncols values.
 *
 * hkb_peer_create allocates this rank's area on `device` (zeroed) and writes
 * its CUDA IPC handle (HKB_PEER_HANDLE_BYTES bytes) to handle_out;
 * hkb_peer_connect opens the other ranks' handles (`handles`: world handles in
 * rank order; this rank's own entry is not read).  `seq` numbers the rounds:
 * 1, 2, 3, ... the same on every rank, skipping multiples of 2^32 (a round's
 * tag is its low 32 bits, and a fresh area holds tag 0).  Every wait is bounded by timeout_ns of
 * the GPU's global timer (0: two seconds); a wait that runs out leaves `out`
 * untouched and sets HKB_PEER_TIMEOUT in the area's status word, which
 * hkb_peer_status reads and clears (a synchronising read).  Before
 * hkb_peer_free, every rank must be past its last hkb_peer_finish (a host
 * barrier): a peer still storing into a freed area would write freed memory. */
#define HKB_PEER_HANDLE_BYTES 64
#define HKB_PEER_MAX_RANKS 8
#define HKB_PEER_TIMEOUT 1u
typedef struct hkb_peer hkb_peer;
int hkb_peer_create(int device, int rank, int world, int dtype, int ncols, hkb_peer** out, void* handle_out);
int hkb_peer_connect(hkb_peer* peer, const void* handles);
int hkb_peer_finish(hkb_peer* peer, int op, void* leaf_hi, void* leaf_comp, int64_t leaves, void* out,
                    uint64_t seq, uint64_t timeout_ns, void* stream);
int hkb_peer_status(hkb_peer* peer, unsigned* flags);
void hkb_peer_free(hkb_peer* peer);

#ifdef __cplusplus
}
#endif

#endif /* HAWK_B200_H */
