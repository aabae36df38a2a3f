/*
 * suika_reshard.h -- C ABI of the B200 live-reshard path.
 *
 * This library replaces the data path of Suika's live state migration:
 *   schedule_param_transfer           Suika/migration.py:322-381  -> rs_plan_build / rs_plan_get_ops
 *   execute_param_transfer            Suika/migration.py:397-556  -> rs_program_build + rs_copy_launch
 *   schedule_and_execute_param_transfer Suika/migration.py:558-598 (the Python mirror in
 *                                     suika_b200/migration.py drives the calls below)
 *   TensorMeta / ParamLayout          Suika/migration.py:29-131, 161-254 -> rs_tensor_meta / rs_rank_layout
 *   TransferOp                        Suika/migration.py:257-312 -> rs_op
 *   dist.isend/irecv per tensor       Suika/utils.py:212-236 -> peer pull through rs_peer_open + rs_copy_launch
 *
 * Conventions
 *   - Every function returns an int status: RS_OK (0) or a negative rs_status code.
 *     rs_last_error() returns a message for the last failure on the calling thread.
 *   - No C++ exception crosses this boundary.
 *   - Plans and programs are immutable after build and may be shared between threads. The only
 *     state kept across calls is the per-thread error message and, for
 *     rs_copy_launch_noalloc, its built-in device table and the per-device address of it.
 *   - Pointers named *_dev are device addresses; everything else is host memory.
 */
#ifndef SUIKA_RESHARD_H
#define SUIKA_RESHARD_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RS_MAX_DIMS 8
/* slice_dim value meaning "tp_meta is None" (tensor replicated across TP). */
#define RS_NO_SLICE (-1000)

enum rs_status {
  RS_OK = 0,
  RS_ERR_ARG = -1,          /* bad argument / malformed descriptor                         */
  RS_ERR_NO_OWNER = -2,     /* "illegal transfer": a target piece has no owner (migration.py:356) */
  RS_ERR_SHAPE = -3,        /* shape / divisibility mismatch (migration.py:293-294,311)      */
  RS_ERR_SLICE_DIM = -4,    /* slice dim mismatch between source and target (migration.py:294, 229) */
  RS_ERR_EMPTY_SOURCE = -5, /* source layout holds no tensor (max() of empty, migration.py:335) */
  RS_ERR_CUDA = -6,         /* a CUDA runtime call failed                                   */
  RS_ERR_BOUNDS = -7,       /* a copy would leave the extent of its source or target        */
  RS_ERR_CAPACITY = -8,     /* caller buffer or workspace too small                         */
  RS_ERR_PEER = -9,         /* peer memory export / import failed                           */
  RS_ERR_SUBFIELD = -10     /* sub-field list inconsistent (migration.py:441)               */
};

/* Cat order of a target tensor assembled from several pieces. */
enum rs_order {
  /* Reproduce the reference: remote pieces in op order, then self pieces in op order
   * (remote pieces are appended while ops are issued, migration.py:472-492; self pieces by the
   * deferred closures, migration.py:448-459 run at :508-509; torch.cat at :536). */
  RS_ORDER_REFERENCE = 0,
  /* Pieces in slice order: the target equals the re-slice of the full tensor. */
  RS_ORDER_SEMANTIC = 1
};

/* Source choice among the owners of a target piece. */
enum rs_src_choice {
  RS_SRC_REFERENCE = 0, /* the reference's greedy rule, migration.py:355-379 */
  RS_SRC_BALANCED = 1   /* least loaded owner by egress bytes, then by rank  */
};

/* One TensorMeta (migration.py:29-131): full (unsharded) shape and TP slicing. */
typedef struct rs_tensor_meta {
  int32_t name_id;              /* index into the caller's name table (shared by all layouts) */
  int32_t ndim;
  int64_t shape[RS_MAX_DIMS];   /* FULL shape: TensorMeta.shape                               */
  int32_t itemsize;             /* bytes per element of TensorMeta.dtype                       */
  int32_t slice_dim;            /* tp_meta[0], or RS_NO_SLICE when tp_meta is None             */
  int32_t tp_index;             /* tp_meta[1]                                                  */
  int32_t tp_deg;               /* tp_meta[2]                                                  */
} rs_tensor_meta;

/* One entry of ParamLayout.layout (migration.py:161-170): rank -> {name -> meta},
 * tensors in the dict's iteration order. Layout arrays list ranks in dict order too. */
typedef struct rs_rank_layout {
  int32_t rank;
  int32_t n_tensors;
  const rs_tensor_meta* tensors;
} rs_rank_layout;

typedef struct rs_plan_opts {
  int32_t minimum_est_peers; /* 1 if IB is enabled else 2 (migration.py:340, utils.py:209-210) */
  int32_t order;             /* enum rs_order                                                  */
  int32_t src_choice;        /* enum rs_src_choice                                             */
  int32_t reserved;
} rs_plan_opts;

/* One TransferOp (migration.py:257-312). The target piece is the rescaled target meta
 * (scale_to_tp, migration.py:103-118); tp fields use RS_NO_SLICE when tp_meta is None. */
typedef struct rs_op {
  int32_t name_id;
  int32_t src_rank;
  int32_t dst_rank;
  int32_t src_slice_dim, src_tp_index, src_tp_deg;
  int32_t dst_slice_dim, dst_tp_index, dst_tp_deg;
  int32_t reserved;
  int64_t numel;               /* elements of the target piece (TensorMeta.numel())            */
} rs_op;

typedef struct rs_plan rs_plan;
typedef struct rs_program rs_program;

const char* rs_last_error(void);
/* 1.1 adds rs_copy_launch_noalloc, rs_act_plan and rs_act_resolve; 1.2 adds rs_copy_run_bounded.
 * The 1.0 entry points are unchanged. */
int rs_version(int32_t* major, int32_t* minor);

/* ---- planning: schedule_param_transfer (migration.py:322-381) -------------------------- */
int rs_plan_build(const rs_rank_layout* src, int32_t n_src,
                  const rs_rank_layout* dst, int32_t n_dst,
                  const rs_plan_opts* opts, rs_plan** out);
int rs_plan_num_ops(const rs_plan* plan, int64_t* n_ops);
int rs_plan_get_ops(const rs_plan* plan, rs_op* ops, int64_t capacity);
void rs_plan_free(rs_plan* plan);

/* ---- layouts the reference does not have ---------------------------------------------------
 * A slice rule describes how a TP shard of one tensor is cut when it is not the reference's
 * contiguous chunk. The slice dim is split into groups (e.g. Q, K, V of a fused QKV weight);
 * group g covers [offset, offset + size) of the full slice dim and consists of `units` equal
 * units (heads). Shard i of degree T holds, group after group, units [i*u/T, (i+1)*u/T) of each
 * group when u >= T, or the single unit floor(i*u/T) when u < T (that unit is then replicated
 * on T/u shards: GQA KV heads at TP above the KV head count). A tensor without a rule is cut into
 * contiguous chunks, as the reference cuts it (Suika/tensor_parallel.py:200-204,378-381).
 *
 * rs_plan_build_rules plans by intersecting the slice intervals of every target shard with those
 * of the source shards (works for any mix of rules and chunks, TP grow and shrink, replicas),
 * writes pieces in slice order, and picks among replicas with the balanced rule. Its targets equal
 * gathering each full tensor from the sources and re-slicing it by the target's rule. */
#define RS_MAX_GROUPS 4

typedef struct rs_slice_group {
  int64_t offset;   /* first index of the group along the slice dim */
  int64_t size;     /* extent of the group along the slice dim     */
  int64_t units;    /* indivisible units (heads) in the group      */
} rs_slice_group;

typedef struct rs_slice_rule {
  int32_t name_id;
  int32_t n_groups;
  rs_slice_group groups[RS_MAX_GROUPS];
} rs_slice_rule;

int rs_plan_build_rules(const rs_rank_layout* src, int32_t n_src,
                        const rs_rank_layout* dst, int32_t n_dst,
                        const rs_slice_rule* rules, int32_t n_rules,
                        const rs_plan_opts* opts, rs_plan** out);

/* ---- per-rank program: the op loop + post-process of execute_param_transfer --------------
 * (migration.py:426-545). For one executing rank it lists the tensors the rank must produce
 * (dst slots), the source tensors it reads (src slots, local or on a peer), the meta
 * (singleton) sub-fields it fills, and the strided copies ("segments") that build every dst
 * slot in place: a TP-grow chunk (get_send_tensor, migration.py:290-312) becomes a row-strided
 * read, a TP-shrink concat (torch.cat, migration.py:536) becomes a row-strided write. */

/* One entry of other_context_dict["expected_sub_fields"] (migration.py:702-709). */
typedef struct rs_subfield {
  int32_t itemsize;   /* bytes per element of this sub-field's tensors          */
  int32_t is_meta;    /* 1: singleton "meta" field (e.g. Adam step), 0: "normal" */
} rs_subfield;

typedef struct rs_program_counts {
  int64_t n_dst_slots;
  int64_t n_src_slots;
  int64_t n_meta_slots;
  int64_t n_segments;
  uint64_t remote_bytes;   /* bytes this rank reads from other ranks           */
  uint64_t local_bytes;    /* bytes this rank copies from its own sources       */
} rs_program_counts;

/* A target tensor to allocate: target_state_dict[name][sub_field]. */
typedef struct rs_dst_slot {
  int32_t name_id;
  int32_t subfield;
  int32_t ndim;
  int32_t reserved;
  int64_t shape[RS_MAX_DIMS];  /* actual (sharded) shape of the target, migration.py:92-98 */
  uint64_t nbytes;
} rs_dst_slot;

/* A source tensor read by this rank: source_state_dict[name][sub_field] on src_rank. */
typedef struct rs_src_slot {
  int32_t src_rank;
  int32_t name_id;
  int32_t subfield;
  int32_t reserved;
  uint64_t nbytes;             /* bytes the source tensor must hold */
} rs_src_slot;

/* A singleton sub-field of a target tensor: its value is the one of the first piece in cat
 * order (tensors[0].clone(), migration.py:538). first_is_self tells which shape the reference
 * gives it: the source tensor's own shape when the first piece is a self transfer
 * (migration.py:446), shape [1] when it was received (migration.py:486-487). */
typedef struct rs_meta_slot {
  int32_t name_id;
  int32_t subfield;
  int32_t src_rank;
  int32_t first_is_self;
} rs_meta_slot;

/* One strided copy: rows x row_bytes from src slot (offset, pitch) to dst slot (offset, pitch). */
typedef struct rs_segment {
  int32_t src_slot;
  int32_t dst_slot;
  uint64_t src_offset;
  uint64_t dst_offset;
  uint64_t rows;
  uint64_t row_bytes;
  uint64_t src_pitch;
  uint64_t dst_pitch;
} rs_segment;

int rs_program_build(const rs_plan* plan, int32_t rank,
                     const rs_subfield* subfields, int32_t n_subfields,
                     rs_program** out);
int rs_program_counts_get(const rs_program* prog, rs_program_counts* out);
int rs_program_dst_slots(const rs_program* prog, rs_dst_slot* out, int64_t capacity);
int rs_program_src_slots(const rs_program* prog, rs_src_slot* out, int64_t capacity);
int rs_program_meta_slots(const rs_program* prog, rs_meta_slot* out, int64_t capacity);
int rs_program_segments(const rs_program* prog, rs_segment* out, int64_t capacity);
void rs_program_free(rs_program* prog);

/* Absolute copy descriptor consumed by the device kernel. */
typedef struct rs_copy_desc {
  uint64_t src_dev;
  uint64_t dst_dev;
  uint64_t rows;
  uint64_t row_bytes;
  uint64_t src_pitch;
  uint64_t dst_pitch;
  uint64_t flags;      /* RS_COPY_REMOTE: source or target is another GPU's memory */
} rs_copy_desc;
#define RS_COPY_REMOTE 1u

/* Bind the program's slots to addresses. src_dev[i]/src_extent[i]: address of src slot i and
 * the bytes readable from it; same for dst. Every segment is checked against the extents
 * (RS_ERR_BOUNDS) before it is written to out[]. Writes rs_program_counts.n_segments entries;
 * entries whose source is another rank get RS_COPY_REMOTE. */
int rs_program_resolve(const rs_program* prog,
                       const uint64_t* src_dev, const uint64_t* src_extent,
                       const uint64_t* dst_dev, const uint64_t* dst_extent,
                       rs_copy_desc* out, int64_t capacity);

/* Like rs_program_resolve, but only for the segments whose source slot lives on `src_rank`
 * (the pieces that rank sends when targets are written by their sources); slots of other ranks
 * may be 0. Writes *n_out entries; RS_COPY_REMOTE when the program's rank is not src_rank. */
int rs_program_resolve_from(const rs_program* prog, int32_t src_rank,
                            const uint64_t* src_dev, const uint64_t* src_extent,
                            const uint64_t* dst_dev, const uint64_t* dst_extent,
                            rs_copy_desc* out, int64_t capacity, int64_t* n_out);

/* ---- device execution (sm_100a) ----------------------------------------------------------
 * One launch executes a whole copy table: local HBM copies and pulls from peer HBM over
 * NVLink alike (a peer address comes from rs_peer_open). Replaces the per-tensor
 * isend/irecv + contiguous/cat/clone of migration.py:466,489,501,536-538. */

typedef struct rs_launch_info {
  uint64_t n_tiles;        /* work units the table was cut into        */
  uint64_t total_bytes;    /* bytes copied                             */
  int64_t n_entries;       /* non-empty entries staged                 */
  uint64_t n_tiles_remote; /* tiles of RS_COPY_REMOTE entries (staged first; every CTA interleaves them
                              with local tiles so NVLink and HBM copies overlap) */
  int32_t grid;            /* CTAs launched                            */
  int32_t block;           /* threads per CTA                          */
  int32_t variant;         /* launch shape (SUIKA_RS_VARIANT - 1)      */
  int32_t reserved;
  /* Tensor-map launch shapes (SUIKA_RS_VARIANT 9-17): the local, 16-byte aligned entries go to a
   * kernel that moves 3-D boxes with cp.async.bulk.tensor (one load and one store per box of
   * whole rows, or up to 2 KB x rows); the fields above then describe the other entries, run by
   * the vector copy. */
  int64_t n_tensor_entries; /* entries (tensor-map pairs) of the tensor-map kernel */
  uint64_t n_tensor_tiles;  /* boxes it moves                                      */
  int32_t tensor_grid;      /* its CTAs                                             */
  int32_t tensor_block;     /* its threads per CTA                                  */
} rs_launch_info;

/* Device workspace the caller must provide to rs_copy_stage / rs_copy_launch for n descriptors
 * (256-byte aligned). It depends on the launch shape SUIKA_RS_VARIANT selects at the time of the
 * call (the tensor-map shapes also stage two 128-byte tensor maps per entry). */
int rs_copy_workspace_bytes(int64_t n_desc, uint64_t* bytes);
/* Cut the table into tiles and stage it into workspace_dev (stream-ordered copy on `stream`, a
 * cudaStream_t; NULL = legacy default stream). Fills *info for rs_copy_run. The launch shape is
 * SUIKA_RS_VARIANT's; unset, a table with no RS_COPY_REMOTE entry takes shape 17 and any other
 * table the vector shape 2. Shapes 15-17 give the local, 16-byte aligned entries with rows wider
 * than 8 KB, and contiguous runs of 1 MB or more, to the tensor-map kernel (17: 3 x 72 KB stages),
 * and the rest to the vector shape 8, in the same run. For the vector shapes, local entries that are column slices of the
 * same source rows (a TP grow's pieces) are cut into row bands of about SUIKA_RS_BAND_BYTES
 * (default 8 MB) per slice and interleaved, so that whole source rows are read at once;
 * rs_launch_info.n_entries counts the entries after that cut. */
int rs_copy_stage(const rs_copy_desc* descs, int64_t n_desc, void* workspace_dev, uint64_t workspace_bytes,
                  void* stream, rs_launch_info* info);
/* Launch the copy kernel over a staged table (asynchronous; may be repeated while the workspace
 * and every address in the table stay valid). Synchronise the stream before reading targets. */
int rs_copy_run(const void* workspace_dev, const rs_launch_info* info, void* stream);
/* rs_copy_run with an explicit bound on every wait inside the kernel. The TMA launch shapes
 * (SUIKA_RS_VARIANT 5-7) wait on shared-memory barriers for their bulk loads; each wait gives up
 * after wait_limit_ns (rs_copy_run uses 2 s), sets status bit 1, drains the copies it issued
 * (bounded again) and ends the CTA, so a stuck copy never hangs the GPU. The vector-copy shapes
 * have no waits. flags: 0, or RS_RUN_STALL_FIRST_STAGE to test that error path (every CTA arms
 * its first stage for bytes that no copy delivers, so that wait runs out; targets stay
 * incomplete); that flag needs a TMA launch shape (else RS_ERR_ARG). */
#define RS_RUN_STALL_FIRST_STAGE 1u
int rs_copy_run_bounded(const void* workspace_dev, const rs_launch_info* info, void* stream,
                        uint64_t wait_limit_ns, uint32_t flags);
/* Status bits of the launches over a staged table since rs_copy_stage cleared them (synchronises
 * `stream`): 0 = no error; 1 = a bounded wait inside the kernel ran out (the kernel stopped
 * early; targets incomplete). */
int rs_copy_status(const void* workspace_dev, const rs_launch_info* info, void* stream, uint32_t* status);
/* rs_copy_stage + rs_copy_run. n_desc == 0 is a no-op. */
int rs_copy_launch(const rs_copy_desc* descs, int64_t n_desc,
                   void* workspace_dev, uint64_t workspace_bytes,
                   void* stream, rs_launch_info* info);

/* ---- copy launch without allocation --------------------------------------------------------
 * No counterpart in the reference. rs_copy_launch needs device workspace for its copy table.
 * Some callers cannot allocate device memory at the moment they reshard. A live migration runs
 * when HBM is fullest: the old and the new layout are both resident, and a framework's caching
 * allocator may already hold the rest of the GPU, so a cudaMalloc can fail or force the
 * allocator to release and synchronise. For them this entry point keeps its copy table in a
 * fixed device array built into the library: at most RS_NOALLOC_MAX_ENTRIES non-empty
 * descriptors per call (about 1.2 MB of device memory, held on every GPU that loads the library
 * until the process exits). It calls no cudaMalloc, cudaFree or other allocating routine.
 *   - Larger tables are rejected with RS_ERR_CAPACITY; use rs_copy_launch for them.
 *   - The first call on a device looks up the array's device address (cudaGetSymbolAddress)
 *     with that device current.
 *   - Every call shares the one array and overwrites the entries it uses; nothing in it needs
 *     to start at zero. Calls on the same stream are ordered; calls that overlap on the GPU
 *     (different streams, or several threads) race on the array.
 *   - It always runs a vector-copy launch shape (SUIKA_RS_VARIANT 1-4 or 8; unset, or a TMA
 *     shape, selects shape 2). Those kernels contain no waits, so a launch cannot stop early and
 *     there is no status word to read back.
 * Otherwise it behaves like rs_copy_launch: same descriptors, same kernel, asynchronous. */
#define RS_NOALLOC_MAX_ENTRIES 16384
int rs_copy_launch_noalloc(const rs_copy_desc* descs, int64_t n_desc, void* stream, rs_launch_info* info);

/* Device address of page-locked host memory (cudaHostAlloc / cudaHostRegister), for copy tables
 * that read host memory directly over PCIe (checkpoint resume, migration.py:1235-1244). */
int rs_host_device_pointer(const void* host_ptr, void** dev_ptr);

/* ---- peer memory (replaces NCCL P2P connections, utils.py:212-236) ----------------------- */
typedef struct rs_peer_handle {
  uint8_t ipc[64];          /* cudaIpcMemHandle_t of the allocation      */
  uint64_t alloc_base;      /* exporter's base address of the allocation */
  uint64_t alloc_bytes;     /* size of the allocation                    */
  int32_t device;           /* exporter's device ordinal                 */
  int32_t pid;              /* exporter's process id                     */
} rs_peer_handle;

/* Export the allocation that contains ptr_dev; *offset = ptr_dev - allocation base. */
int rs_peer_export(const void* ptr_dev, rs_peer_handle* out, uint64_t* offset);
/* Map a peer's exported allocation into this process (current device); *base_dev is the
 * local address of the allocation base. Close with rs_peer_close after every reader is done. */
int rs_peer_open(const rs_peer_handle* handle, void** base_dev);
int rs_peer_close(void* base_dev);

/* ---- activation exchange between pipeline stages ----------------------------------------
 * Replaces the cross-stage send/recv of PipelineExecModule (Suika/pipeline_parallel.py:665-836):
 * per rank, a list of P2P ops built by _get_recv_or_send_P2P_ops (:665-776), each staging a
 * .contiguous() copy of a (batch range x slice chunk) block (:748-756) and copying it back after
 * the transfer, followed on the receive side by a TP all-gather and a cat (:817-832). Here every
 * receiver's complete tensor is planned as pieces that one copy launch (rs_copy_launch) writes
 * straight into place: no staging copies, no all-gather, no cat. Bytes written are the ones the
 * reference delivers, from the same sender. */

/* One stage's DeviceMesh2D (Suika/device_mesh.py:150-240) with its local batch sizes
 * (lbsz_mesh[stage], pipeline_parallel.py:175): DP group g is the TP group
 * ranks[group_start[g] .. group_start[g + 1]); groups hold batch rows in group order. */
typedef struct rs_stage_mesh {
  int32_t n_groups;
  int32_t reserved;
  const int32_t* group_start; /* n_groups + 1 offsets into ranks   */
  const int32_t* ranks;
  const int64_t* local_bsz;   /* local batch size of each DP group */
} rs_stage_mesh;

/* One block a receiver gets: batch rows [dst_batch, dst_batch + n_batch) of its local tensor
 * (rows [src_batch, ...) of the sender's) by slice-dim range [slice_start, slice_start + slice_len). */
typedef struct rs_act_piece {
  int32_t src_rank;
  int32_t dst_rank;
  int64_t src_batch;
  int64_t dst_batch;
  int64_t n_batch;
  int64_t slice_start;
  int64_t slice_len;
} rs_act_piece;

/* Layout of every rank's activation tensor (contiguous, row-major). shape[batch_dim] is ignored:
 * each rank's own local batch size applies. batch_dim and slice_dim are non-negative and differ. */
typedef struct rs_act_geometry {
  int32_t ndim;
  int32_t batch_dim;
  int32_t slice_dim;
  int32_t elem_bytes;
  int64_t shape[RS_MAX_DIMS];
} rs_act_geometry;

/* Every piece from stage src to stage dst, receiver by receiver (DP group, then TP index), then
 * sending DP group, then slice position. Sends only where the batch ranges overlap
 * (pipeline_parallel.py:711-721). Along the slice dim an overlap is cut into k = max(s, d)
 * chunks, s and d the two groups' TP degrees (powers of two, else RS_ERR_SHAPE); chunk c comes
 * from TP rank c * s / k of the sending group. slice_size % k != 0 is RS_ERR_SHAPE. out == NULL
 * only counts: *n_out = number of pieces. */
int rs_act_plan(const rs_stage_mesh* src, const rs_stage_mesh* dst, int64_t slice_size,
                rs_act_piece* out, int64_t capacity, int64_t* n_out);

/* Copy descriptors of pieces. src_dev[r] / dst_dev[r]: base address of rank r's sending /
 * receiving tensor in this process (r < n_ranks; a piece whose address is 0 is RS_ERR_ARG).
 * A piece becomes prod(shape[:min(batch_dim, slice_dim)]) descriptors; pieces that leave a
 * rank's tensor are RS_ERR_BOUNDS. RS_COPY_REMOTE is set when the two ranks differ. out == NULL
 * only counts. */
int rs_act_resolve(const rs_stage_mesh* src, const rs_stage_mesh* dst, const rs_act_geometry* geometry,
                   const rs_act_piece* pieces, int64_t n_pieces,
                   const uint64_t* src_dev, const uint64_t* dst_dev, int32_t n_ranks,
                   rs_copy_desc* out, int64_t capacity, int64_t* n_out);

#ifdef __cplusplus
}
#endif
#endif /* SUIKA_RESHARD_H */
