/* eagle_b200: a B200 (sm_100a) backend for eagle's until-done hot path, behind
 * eagle's ``eagle-backend/1`` C seam.
 *
 * Every declaration below is ``extern "C"``, takes plain pointers, integers and
 * POD descs (no C++ or torch types), and keeps the name, argument meaning, struct
 * layout and status behaviour of the seam entry it replaces. Each carries the
 * reference declaration it stands in for as ``python/src/seam/eagle_backend.h:LINE``
 * (paths relative to the eagle source tree). Entries named ``eagle_backend_x_b200_*``
 * are this backend's own additions; each says so.
 *
 * Conventions (eagle_backend.h:59-88): every desc starts with ``uint32_t
 * struct_size``; an input desc is read up to min(caller, callee) size, the rest
 * taken as zero; unknown flag bits return EAGLE_BACKEND_UNSUPPORTED; ``device ==
 * -1`` is the device owning the desc's buffers (else the current one); a raw
 * stream 0 is the legacy default stream; a non-OK status leaves its message in
 * the calling thread's ``eagle_backend_last_error()``, valid until the next call.
 */
#ifndef EAGLE_B200_H
#define EAGLE_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- versions, statuses, capability bits (eagle_backend.h:104-141) ---------- */

#define EAGLE_BACKEND_VERSION_MAJOR 1u
#define EAGLE_BACKEND_VERSION_MINOR 8u
#define EAGLE_BACKEND_VERSION ((EAGLE_BACKEND_VERSION_MAJOR << 16) | EAGLE_BACKEND_VERSION_MINOR)

typedef int32_t eagle_backend_status;

#define EAGLE_BACKEND_OK 0
#define EAGLE_BACKEND_ERROR 1
#define EAGLE_BACKEND_INVALID_ARGUMENT 2
#define EAGLE_BACKEND_INDEX 3
#define EAGLE_BACKEND_INTEROP 4
#define EAGLE_BACKEND_UNAVAILABLE 5
#define EAGLE_BACKEND_CALLBACK_FAILED 6
#define EAGLE_BACKEND_BAD_HANDLE 7
#define EAGLE_BACKEND_UNSUPPORTED 8

#define EAGLE_BACKEND_CAP_STREAM (UINT64_C(1) << 0)
#define EAGLE_BACKEND_CAP_CAPTURER (UINT64_C(1) << 1)
#define EAGLE_BACKEND_CAP_CAPTURED (UINT64_C(1) << 2)
#define EAGLE_BACKEND_CAP_FORK (UINT64_C(1) << 3)
#define EAGLE_BACKEND_CAP_CONDITIONAL (UINT64_C(1) << 4)
#define EAGLE_BACKEND_CAP_ATTRIBUTION (UINT64_C(1) << 5)
#define EAGLE_BACKEND_CAP_GRAPH (UINT64_C(1) << 6)
#define EAGLE_BACKEND_CAP_LAUNCHER (UINT64_C(1) << 7)
#define EAGLE_BACKEND_CAP_EXEC (UINT64_C(1) << 9)
#define EAGLE_BACKEND_CAP_DEVICE (UINT64_C(1) << 10)
#define EAGLE_BACKEND_CAP_INTEROP (UINT64_C(1) << 11)
#define EAGLE_BACKEND_CAP_FILTERING (UINT64_C(1) << 12)
#define EAGLE_BACKEND_CAP_CONDITIONAL_IF_ELSE (UINT64_C(1) << 13)
#define EAGLE_BACKEND_CAP_CONDITIONAL_SWITCH (UINT64_C(1) << 14)

/* Conditional node kinds (eagle_backend.h:144-147); 0 = WHILE when counter_ptr
 * is set, else IF. */
#define EAGLE_BACKEND_COND_IF 1u
#define EAGLE_BACKEND_COND_IF_ELSE 2u
#define EAGLE_BACKEND_COND_WHILE 3u
#define EAGLE_BACKEND_COND_SWITCH 4u
/* A WHILE's loop_cap for a loop the guard alone ends. */
#define EAGLE_BACKEND_LOOP_UNCAPPED 0xFFFFFFFFu

typedef struct eagle_backend_stream_s* eagle_backend_stream;
typedef struct eagle_backend_capturer_s* eagle_backend_capturer;
typedef struct eagle_backend_captured_s* eagle_backend_captured;
typedef struct eagle_backend_fork_s* eagle_backend_fork;
typedef struct eagle_backend_conditional_s* eagle_backend_conditional;
typedef struct eagle_backend_graph_s* eagle_backend_graph;
typedef struct eagle_backend_launcher_s* eagle_backend_launcher;

/* ---- structs ------------------------------------------------------------------ */

/* eagle_backend.h:171-179 */
struct eagle_backend_build_info {
    uint32_t struct_size;
    uint32_t abi_version;
    int32_t cudart_version;
    int32_t reserved0;
    char eagle_version[32];
    char archs[128];
    char backend_kind[16];
};

/* eagle_backend.h:181-192 */
struct eagle_backend_device_props {
    uint32_t struct_size;
    int32_t device;
    char name[256];
    int32_t cc_major, cc_minor, sm_count, clock_rate_khz, memory_clock_rate_khz, memory_bus_width_bits;
    int32_t regs_per_block, regs_per_sm, warp_size, reserved0;
    int64_t shared_mem_per_block, shared_mem_per_sm;
    double peak_bytes_per_s, peak_flops_sp, peak_flops_dp, fp64_ratio;
    double ridge_flops_per_byte_sp, ridge_flops_per_byte_dp;
    int64_t total_mem_bytes, free_mem_bytes;
};

/* eagle_backend.h:194-199 */
struct eagle_backend_stream_desc {
    uint32_t struct_size;
    uint32_t flags;
    int32_t device;
    int32_t reserved0;
};

/* eagle_backend.h:200-206 */
struct eagle_backend_capturer_desc {
    uint32_t struct_size;
    uint32_t flags;
    int32_t device;
    int32_t reserved0;
    uint64_t stream; /* the stream to capture */
};

/* eagle_backend.h:208-216 */
struct eagle_backend_fork_desc {
    uint32_t struct_size;
    uint32_t flags;
    int32_t device;
    int32_t reserved0;
    uint64_t origin;       /* the stream the branches fork from */
    uint64_t branch_count;
    uint64_t wait_count;   /* marks fork_mark may make */
};

/* eagle_backend.h:218-234. The guard is ``(*count != (baseline ? *baseline : 0))
 * != negate`` (a null count always holds); a WHILE keeps ``counter_ptr[2] =
 * {remaining, ran}``, reset by its head setter every replay. */
struct eagle_backend_conditional_desc {
    uint32_t struct_size;
    uint32_t flags;
    int32_t device;
    uint32_t loop_cap;     /* WHILE iteration cap per replay, >= 1 */
    uint64_t origin;       /* the capturing stream the node is woven into */
    uint64_t count_ptr;    /* device uint32* (SWITCH: the arm index) */
    uint64_t baseline_ptr; /* device uint32*, 0 = none */
    uint64_t counter_ptr;  /* device uint32[2] for a WHILE, 0 = IF */
    uint32_t kind;         /* EAGLE_BACKEND_COND_*, 0 = from counter_ptr */
    uint32_t arms;         /* 0 = the kind's own; SWITCH: the arm count */
    uint32_t negate;
    uint32_t reserved1;
    uint64_t brk_ptr;      /* WHILE: device uint32 break cell, 0 = none */
    uint64_t limit_ptr;    /* WHILE: device uint32 trip count, 0 = none */
};

/* eagle_backend.h:236-241 */
struct eagle_backend_graph_desc {
    uint32_t struct_size;
    uint32_t flags;
    int32_t device;
    int32_t reserved0;
};
#define EAGLE_BACKEND_STREAM_NON_BLOCKING 1u

/* eagle_backend.h:244-256: one kernel launch over one partition */
struct eagle_backend_launch_desc {
    uint32_t struct_size;
    uint32_t flags;
    int32_t device;
    uint32_t block;
    uint64_t function;
    const uint64_t* params;
    const uint64_t* param_sizes;
    int64_t nparams;
    int64_t base, count, n_samples;
    uint64_t stream;
};

/* eagle_backend.h:480-493 */
struct eagle_backend_launch_raw_desc {
    uint32_t struct_size;
    uint32_t flags;
    int32_t device;
    uint32_t shared_bytes;
    uint64_t function;
    uint64_t stream;
    uint32_t grid[3];
    uint32_t block[3];
    uint64_t args;
    uint32_t arg_count;
    uint32_t reserved;
};

/* cell ops (eagle_backend.h:497-523): integer kernels, bit-equal to the plain C expression */
#define EAGLE_BACKEND_CELL_BUMP 0u
#define EAGLE_BACKEND_CELL_MASK_COUNT 1u
#define EAGLE_BACKEND_CELL_POLICY 2u
#define EAGLE_BACKEND_CELL_IDENTITY 3u
#define EAGLE_BACKEND_CELL_COUNT_FIRED 4u
#define EAGLE_BACKEND_CELL_GROUP_AND 5u
#define EAGLE_BACKEND_CELL_SCALE_COUNT 6u

/* eagle_backend.h:576-587 */
struct eagle_backend_cell_op_desc {
    uint32_t struct_size;
    uint32_t flags;
    uint32_t op;
    int32_t device;
    uint64_t stream;
    int64_t n;
    uint64_t p[6];
    int64_t i[10];
    double f[2];
    int64_t j[4];
};

/* filtering (eagle_backend.h:666-691) */
#define EAGLE_BACKEND_COMPACT_MASK_IS_DROP (UINT32_C(1) << 0)

struct eagle_backend_compact_desc {
    uint32_t struct_size;
    uint32_t flags;
    int32_t device;
    uint32_t reserved;
    uint64_t mask;
    uint64_t index_map;
    uint64_t count;
    uint64_t scratch;
    int64_t n;
    uint64_t stream;
    int64_t scratch_bytes;
    uint64_t live32;
    uint64_t span;
    uint64_t fire;
    float theta;
    uint32_t reserved2;
};

/* eagle_backend.h:705-730 (reset_device reads device, perm, inv, index_map, count, span, n, stream) */
struct eagle_backend_reorder_plane {
    uint64_t data;
    uint32_t elem_bytes;
    uint32_t reserved;
};

struct eagle_backend_reorder_desc {
    uint32_t struct_size;
    uint32_t flags;
    int32_t device;
    uint32_t n_planes;
    uint64_t planes;
    uint64_t mask;
    uint64_t perm;
    uint64_t inv;
    uint64_t index_map;
    uint64_t count;
    uint64_t span;
    uint64_t fire;
    uint64_t scratch;
    int64_t n;
    uint64_t stream;
    int64_t scratch_bytes;
};

/* canonical reduction (eagle_backend.h:861-894) */
#define EAGLE_BACKEND_REDUCE_F32 0u
#define EAGLE_BACKEND_REDUCE_F64 1u
#define EAGLE_BACKEND_REDUCE_I32 2u
#define EAGLE_BACKEND_REDUCE_I64 3u
#define EAGLE_BACKEND_REDUCE_U8 4u
#define EAGLE_BACKEND_REDUCE_OP_SUM 0u
#define EAGLE_BACKEND_REDUCE_OP_MAX 1u
#define EAGLE_BACKEND_REDUCE_OP_ALL 2u
#define EAGLE_BACKEND_REDUCE_OP_MIN 3u
#define EAGLE_BACKEND_REDUCE_COMPENSATED 0u
#define EAGLE_BACKEND_REDUCE_ORDERED 1u
#define EAGLE_BACKEND_REDUCE_AUTO 2u
#define EAGLE_BACKEND_REDUCE_PAIR_OUT 1u

struct eagle_backend_reduce_desc {
    uint32_t struct_size;
    uint32_t dtype;
    uint32_t op;
    int32_t device;
    uint64_t in;
    uint64_t out;
    uint64_t work_a;
    uint64_t work_b;
    int64_t n;
    uint64_t stream;
    int64_t work_elems;
    uint32_t policy;
    uint32_t flags;
    int64_t columns;
    uint64_t comp_in;
};

/* ---- mandatory core (eagle_backend.h:268-277) --------------------------------- */

/* eagle_backend.h:268: (1 << 16) | 8 */
uint32_t eagle_backend_version(void);
/* eagle_backend.h:269: the calling thread's message of its last failed call */
const char* eagle_backend_last_error(void);
/* eagle_backend.h:270 */
eagle_backend_status eagle_backend_build_info(struct eagle_backend_build_info* info);
/* eagle_backend.h:272: OK when a CUDA device is usable, UNAVAILABLE otherwise */
eagle_backend_status eagle_backend_probe(void);
/* eagle_backend.h:273: frees a buffer this backend allocated (NULL-safe) */
void eagle_backend_free(void* p);
/* eagle_backend.h:274 */
eagle_backend_status eagle_backend_capabilities(uint64_t* groups);
/* eagle_backend.h:277: the DLPack device types served (kDLCUDA = 2) */
eagle_backend_status eagle_backend_device_types(int32_t* types, int32_t cap, int32_t* count);

/* ---- stream (bit 0; eagle_backend.h:281-284) ---------------------------------- */

eagle_backend_status eagle_backend_stream_create(const struct eagle_backend_stream_desc* desc, eagle_backend_stream* out);
eagle_backend_status eagle_backend_stream_ptr(eagle_backend_stream h, uint64_t* stream);
eagle_backend_status eagle_backend_stream_synchronize(eagle_backend_stream h);
void eagle_backend_stream_release(eagle_backend_stream h);

/* ---- capturer (bit 1; eagle_backend.h:288-294): a thread-local stream capture - */

eagle_backend_status eagle_backend_capturer_create(const struct eagle_backend_capturer_desc* desc, eagle_backend_capturer* out);
eagle_backend_status eagle_backend_capturer_begin(eagle_backend_capturer h);
eagle_backend_status eagle_backend_capturer_end(eagle_backend_capturer h, eagle_backend_captured* out);
/* eagle_backend.h:292: the graph the in-flight capture records into (0: none) */
eagle_backend_status eagle_backend_capturer_graph(eagle_backend_capturer h, uint64_t* graph);
void eagle_backend_capturer_release(eagle_backend_capturer h);

/* ---- captured (bit 2; eagle_backend.h:298-299) --------------------------------- */

eagle_backend_status eagle_backend_captured_is_valid(eagle_backend_captured h, int32_t* valid);
void eagle_backend_captured_release(eagle_backend_captured h);

/* ---- fork (bit 3; eagle_backend.h:303-318): branch streams made at create ------ */

eagle_backend_status eagle_backend_fork_create(const struct eagle_backend_fork_desc* desc, eagle_backend_fork* out);
eagle_backend_status eagle_backend_fork_fork(eagle_backend_fork h);
eagle_backend_status eagle_backend_fork_join(eagle_backend_fork h);
/* INDEX when ``i`` is out of range */
eagle_backend_status eagle_backend_fork_branch(eagle_backend_fork h, uint64_t i, uint64_t* stream);
eagle_backend_status eagle_backend_fork_origin(eagle_backend_fork h, uint64_t* stream);
eagle_backend_status eagle_backend_fork_forked(eagle_backend_fork h, int32_t* forked);
eagle_backend_status eagle_backend_fork_size(eagle_backend_fork h, uint64_t* n);
void eagle_backend_fork_release(eagle_backend_fork h);
/* eagle_backend.h:314-318: mark branch ``producer``'s tip; branch ``waiter`` waits on a mark */
eagle_backend_status eagle_backend_fork_mark(eagle_backend_fork h, uint64_t producer, uint64_t* mark);
eagle_backend_status eagle_backend_fork_wait(eagle_backend_fork h, uint64_t waiter, uint64_t mark);

/* ---- conditional (bit 4, + 13 IF/ELSE, 14 SWITCH; eagle_backend.h:322-333) -----
 * create makes the arm streams (call it before the capture begins); begin weaves a
 * 1x1 setter kernel and the conditional node at the origin's capture tip and opens
 * the arm captures; end closes them (a WHILE first captures its tail setter as the
 * body's last node). An arm that launched nothing is refused at end. */

eagle_backend_status eagle_backend_conditional_create(const struct eagle_backend_conditional_desc* desc, eagle_backend_conditional* out);
eagle_backend_status eagle_backend_conditional_begin(eagle_backend_conditional h, uint64_t* body_stream);
eagle_backend_status eagle_backend_conditional_body_stream(eagle_backend_conditional h, uint64_t* body_stream);
eagle_backend_status eagle_backend_conditional_is_loop(eagle_backend_conditional h, int32_t* is_loop);
eagle_backend_status eagle_backend_conditional_end(eagle_backend_conditional h);
void eagle_backend_conditional_release(eagle_backend_conditional h);
eagle_backend_status eagle_backend_conditional_arm_stream(eagle_backend_conditional h, uint64_t k, uint64_t* stream);
/* ``which`` >= 0: arm ``which``'s body nodes; -1: the setter nodes (head, + a
 * WHILE's tail). ``*nodes`` is freed with eagle_backend_free. */
eagle_backend_status eagle_backend_conditional_nodes(eagle_backend_conditional h, int64_t which, uint64_t** nodes,
    int64_t* count);

/* ---- attribution (bit 5; eagle_backend.h:339-346) ------------------------------ */

eagle_backend_status eagle_backend_capture_snapshot_nodes(uint64_t stream, uint64_t** nodes, int64_t* count);
eagle_backend_status eagle_backend_is_node_toggleable(uint64_t node, int32_t* toggleable);
eagle_backend_status eagle_backend_capture_add_child(uint64_t stream, uint64_t child, int32_t conditional_body);

/* ---- graph (bit 6; eagle_backend.h:350-358): a created graph starts with one
 * empty node; add_node chains a captured graph after the last node -------------- */

eagle_backend_status eagle_backend_graph_create(const struct eagle_backend_graph_desc* desc, eagle_backend_graph* out);
/* CONSUMES ``captured`` on OK; INVALID_ARGUMENT for an empty capture */
eagle_backend_status eagle_backend_graph_from_captured(eagle_backend_captured captured, eagle_backend_graph* out);
eagle_backend_status eagle_backend_graph_stream(eagle_backend_graph h, uint64_t stream);
/* CONSUMES ``captured`` on OK */
eagle_backend_status eagle_backend_graph_add_node(eagle_backend_graph h, eagle_backend_captured captured);
eagle_backend_status eagle_backend_graph_launcher(eagle_backend_graph h, eagle_backend_launcher* out);
eagle_backend_status eagle_backend_graph_last_node(eagle_backend_graph h, int64_t* index);
void eagle_backend_graph_release(eagle_backend_graph h);

/* ---- launcher (bit 7; eagle_backend.h:362-383): an instantiated graph ---------- */

eagle_backend_status eagle_backend_launcher_launch(eagle_backend_launcher h);
eagle_backend_status eagle_backend_launcher_synchronize(eagle_backend_launcher h);
eagle_backend_status eagle_backend_launcher_stream(eagle_backend_launcher h, uint64_t stream);
/* Re-grid every kernel node add_node gathered to ceil(logical_size / block); 0 keeps them */
eagle_backend_status eagle_backend_launcher_set_logical_size(eagle_backend_launcher h, int64_t logical_size);
eagle_backend_status eagle_backend_launcher_kernel_node_count(eagle_backend_launcher h, int64_t* count);
eagle_backend_status eagle_backend_launcher_set_node_enabled(eagle_backend_launcher h, uint64_t node, int32_t enabled);
void eagle_backend_launcher_release(eagle_backend_launcher h);
/* Patch kernel node ``node``'s first ``n`` arguments from ``params`` (0 keeps the
 * captured value); the source graph's node is patched too */
eagle_backend_status eagle_backend_launcher_set_kernel_params(eagle_backend_launcher h, uint64_t node,
    const uint64_t* params, int64_t n);
eagle_backend_status eagle_backend_launcher_set_memcpy_source(eagle_backend_launcher h, uint64_t node, uint64_t src);
/* ``*accepted`` = 0 when the driver rejects the update (the exec is unchanged) */
eagle_backend_status eagle_backend_launcher_exec_update(eagle_backend_launcher h, eagle_backend_captured captured,
    int32_t* accepted);
/* An owned clone of the source graph (a cudaGraph_t); refuses host-function,
 * conditional and memory-allocation nodes */
eagle_backend_status eagle_backend_launcher_clone_graph(eagle_backend_launcher h, uint64_t* graph);
eagle_backend_status eagle_backend_launcher_graph_destroy(uint64_t graph);

/* ---- exec (bit 9; eagle_backend.h:389) ----------------------------------------- */

/* One launch of ``desc->function`` over the partition (base, count, n_samples): the
 * packed role arguments, then the partition triple appended by value (the hawk
 * kernel ABI, eagle/exec/DeviceKernel.h:47-84); grid = ceil(count / block).
 * ``*launched`` = 0 for an empty partition. */
eagle_backend_status eagle_backend_run_device(const struct eagle_backend_launch_desc* desc, int32_t* launched);

/* ---- device (bit 10; eagle_backend.h:393) -------------------------------------- */

eagle_backend_status eagle_backend_device_props(int32_t device, struct eagle_backend_device_props* props);

/* ---- interop (bit 11; eagle_backend.h:396-440) --------------------------------- */

/* eagle_backend.h:150: "no stream given" in a fence stream argument */
#define EAGLE_BACKEND_STREAM_NONE INT64_MIN
/* eagle_backend.h:399: order everything queued on ``producer`` before what is queued
 * later on ``consumer`` (DLPack stream codes: 1 legacy default, 2 per-thread default,
 * -1 no ordering, 0 refused, else a raw stream), without blocking the host */
eagle_backend_status eagle_backend_fence(int32_t dl_device_type, int32_t device_id, int64_t producer, int64_t consumer);
/* eagle_backend.h:400: events the fence pool has created */
eagle_backend_status eagle_backend_event_pool_created(int64_t* count);
/* eagle_backend.h:429-433: page-locked host memory the device can DMA from (0 for 0 bytes) */
eagle_backend_status eagle_backend_host_alloc(uint64_t bytes, uint64_t* out);
eagle_backend_status eagle_backend_host_free(uint64_t ptr);
/* eagle_backend.h:438-440: call fn(arg) once the work enqueued before it on ``stream``
 * is done; capture-legal (a host node); fn must not call the backend */
eagle_backend_status eagle_backend_host_func(uint64_t stream, void (*fn)(void*), void* arg);

/* ---- memory, per symbol (eagle_backend.h:405-424) ------------------------------ */

#define EAGLE_BACKEND_COPY_H2D 0
#define EAGLE_BACKEND_COPY_D2H 1
#define EAGLE_BACKEND_COPY_D2D 2
#define EAGLE_BACKEND_COPY_H2H 3

/* eagle_backend.h:405: zero ``bytes`` at device ``ptr`` on ``stream`` (capture-legal) */
eagle_backend_status eagle_backend_memset_device(uint64_t ptr, uint64_t bytes, uint64_t stream);
/* eagle_backend.h:409 */
eagle_backend_status eagle_backend_memcpy_device(uint64_t dst, uint64_t src, uint64_t bytes, uint64_t stream);
/* eagle_backend.h:424 */
eagle_backend_status eagle_backend_memcpy(uint64_t dst, uint64_t src, uint64_t bytes, int32_t kind, uint64_t stream);

/* ---- device scope, raw launch, cell ops, events (minor 7; eagle_backend.h:442-662) */

/* eagle_backend.h:442 */
eagle_backend_status eagle_backend_device_count(int32_t* count);
/* eagle_backend.h:444 */
eagle_backend_status eagle_backend_set_device(int32_t device);
/* eagle_backend.h:447 */
eagle_backend_status eagle_backend_get_device(int32_t* device);
/* eagle_backend.h:451: read and clear the thread's pending launch error */
eagle_backend_status eagle_backend_launch_status(int32_t device);
/* eagle_backend.h:453 */
eagle_backend_status eagle_backend_device_synchronize(int32_t device);
/* eagle_backend.h:455 */
eagle_backend_status eagle_backend_stream_is_capturing(uint64_t stream, int32_t* capturing);
/* eagle_backend.h:461: load a cubin, fatbin or PTX image in the primary context of
 * ``device`` (-1: the current one) -- how a hawk artifact's kernels arrive */
eagle_backend_status eagle_backend_module_load(const void* image, uint64_t bytes, int32_t device, uint64_t* module);
/* eagle_backend.h:464: module_load of PTX under a cap of max_registers per thread (0: none) */
eagle_backend_status eagle_backend_module_load_jit(const void* image, uint64_t bytes, int32_t device,
    uint32_t max_registers, uint64_t* module);
/* eagle_backend.h:469: link PTX for ``device`` and copy the cubin to ``out`` (null: size only) */
eagle_backend_status eagle_backend_link_ptx(const void* image, uint64_t bytes, int32_t device, uint32_t max_registers,
    void* out, uint64_t capacity, uint64_t* size);
/* eagle_backend.h:473: the function ``name`` of ``module`` (INDEX when absent) */
eagle_backend_status eagle_backend_module_function(uint64_t module, const char* name, uint64_t* function);
/* eagle_backend.h:475 */
void eagle_backend_module_release(uint64_t module, int32_t device);
/* eagle_backend.h:622: cudaMemcpy2DAsync of ``height`` rows of ``width_bytes`` (not H2H) */
eagle_backend_status eagle_backend_memcpy_strided(uint64_t dst, uint64_t dst_pitch, uint64_t src, uint64_t src_pitch,
    uint64_t width_bytes, uint64_t height, int32_t kind, uint64_t stream);

/* eagle_backend.h:627-644: stream-ordered memory (eagle's array layer) */
#define EAGLE_BACKEND_MEM_DEVICE 0
#define EAGLE_BACKEND_MEM_PINNED 1
/* a device allocation is stream-ordered on ``stream`` and 256-byte aligned; refused
 * while the stream is capturing; bytes == 0 gives null ptr and chunk */
eagle_backend_status eagle_backend_mem_alloc(int32_t kind, int32_t device, uint64_t bytes, uint64_t stream,
    uint64_t* chunk, uint64_t* ptr);
/* stream-ordered free; deferred while the allocation stream is capturing */
void eagle_backend_mem_release(uint64_t chunk);
/* run the deferred frees; ``*left`` (may be null) = frees still queued */
eagle_backend_status eagle_backend_mem_drain(int64_t* left);
/* the device of the allocation holding ``ptr`` (-1: host or unknown) */
eagle_backend_status eagle_backend_pointer_device(uint64_t ptr, int32_t* device);
/* eagle_backend.h:478: one CUfunction attribute (cuFuncGetAttribute codes) */
eagle_backend_status eagle_backend_function_attribute(uint64_t function, int32_t attribute, int32_t* value);
/* eagle_backend.h:495: cuLaunchKernel of desc->function; enqueue only, capture-legal */
eagle_backend_status eagle_backend_launch_raw(const struct eagle_backend_launch_raw_desc* desc);
/* eagle_backend.h:590: ops BUMP, MASK_COUNT, POLICY, IDENTITY, COUNT_FIRED,
 * GROUP_AND, SCALE_COUNT (the until-done loop's ops); the array ops 7-35 return
 * UNSUPPORTED. Capture-legal: enqueue only. */
eagle_backend_status eagle_backend_cell_op(const struct eagle_backend_cell_op_desc* desc);
/* eagle_backend.h:648 */
eagle_backend_status eagle_backend_stream_sync(int32_t device, uint64_t stream);
/* eagle_backend.h:651-662 */
eagle_backend_status eagle_backend_event_create(int32_t device, uint64_t* event);
eagle_backend_status eagle_backend_event_create_timed(int32_t device, uint64_t* event);
eagle_backend_status eagle_backend_event_elapsed(uint64_t start, uint64_t end, float* ms);
eagle_backend_status eagle_backend_event_record(uint64_t event, uint64_t stream);
eagle_backend_status eagle_backend_event_wait(uint64_t stream, uint64_t event);
void eagle_backend_event_release(uint64_t event, int32_t device);

/* ---- filtering (bit 12; eagle_backend.h:701, :832) ----------------------------- */

/* eagle_backend.h:693-701: compact the samples ``mask`` keeps into
 * index_map[0, *count), ascending. ``scratch == 0`` is the query (writes
 * scratch_bytes only). Otherwise enqueue only: no allocation, no synchronisation,
 * no host read (capturable). n > 2^31 - 1 returns UNSUPPORTED. One single-pass
 * kernel (warp ballots, decoupled look-back) after a memset of its scratch. */
eagle_backend_status eagle_backend_compact_device(struct eagle_backend_compact_desc* desc);
/* eagle_backend.h:826-832: perm, inv and (non-zero) index_map become 0..n-1,
 * *count = *span = n, in one kernel; capture-legal */
eagle_backend_status eagle_backend_reset_device(struct eagle_backend_reorder_desc* desc);
/* eagle_backend.h:705-740: permute every plane IN PLACE over [0, *span) so the kept
 * samples fill [0, *count) in ascending sample order and the dropped ones follow in
 * ascending order; perm moves with them, inv is rebuilt for the moved slots,
 * index_map becomes the identity over [0, *count), *span = *count. The mask is one
 * of the planes. With fire != 0 every kernel returns while *fire == 0 and the last
 * clears it. Query with scratch == 0 (scratch_bytes). Enqueue only, capturable. */
eagle_backend_status eagle_backend_reorder_device(struct eagle_backend_reorder_desc* desc);
/* eagle_backend.h:855-859: undo every reorder since the last restore: each plane back
 * in sample order, perm and inv the identity (mask, index_map, count, span and fire
 * are not read). Query with scratch == 0. Enqueue only. */
eagle_backend_status eagle_backend_x_restore_device(struct eagle_backend_reorder_desc* desc);

/* ---- filtering: K classes (eagle_backend.h:742-824) ---------------------------- */

/* reorder_classes flags: sort [0, *count) by class only (the live prefix) */
#define EAGLE_BACKEND_CLASSES_WITHIN_LIVE (UINT32_C(1) << 1)
#define EAGLE_BACKEND_MAX_CLASSES 255

/* eagle_backend.h:755-781: compact_device plus the K-class trigger; live32, span and
 * fire are required here */
struct eagle_backend_compact_classes_desc {
    uint32_t struct_size;
    uint32_t flags;
    int32_t device;
    uint32_t reserved;
    uint64_t mask;
    uint64_t index_map;
    uint64_t count;
    uint64_t scratch;
    int64_t n;
    uint64_t stream;
    int64_t scratch_bytes;
    uint64_t live32;
    uint64_t span;
    uint64_t fire;
    float theta;
    uint32_t reserved2;
    uint64_t class_plane;   /* uint8_t[n], each sample's class in [0, classes) */
    uint32_t classes;       /* K, in [2, 255] */
    float class_theta;      /* the mixed-group threshold, in (0, 1) */
    uint64_t offsets;       /* not written here */
    uint64_t mixed32;       /* uint32_t[1]: OUT, 32-slot groups holding two or more live classes */
    uint64_t stale_count;   /* uint32_t[1]: IN, samples whose class changed since the last sort; 0 = none */
    uint64_t class_fire;    /* uint32_t[1]: OUT, (mixed32 > 0 && mixed32 >= class_theta * live32 &&
                             * span >= 4096) || stale_count > 0.05 * count || fire */
    uint64_t reserved3;
};

/* eagle_backend.h:787: compaction with the class trigger (query and capture as compact_device) */
eagle_backend_status eagle_backend_compact_classes_device(struct eagle_backend_compact_classes_desc* desc);

/* eagle_backend.h:792-812: reorder_device generalised to K classes */
struct eagle_backend_reorder_classes_desc {
    uint32_t struct_size;
    uint32_t flags;         /* COMPACT_MASK_IS_DROP | CLASSES_WITHIN_LIVE */
    int32_t device;
    uint32_t n_planes;
    uint64_t planes;
    uint64_t mask;
    uint64_t perm;
    uint64_t inv;
    uint64_t index_map;
    uint64_t count;
    uint64_t span;
    uint64_t fire;
    uint64_t scratch;
    int64_t n;
    uint64_t stream;
    int64_t scratch_bytes;
    uint64_t class_plane;   /* uint8_t[n], one of the planes */
    uint32_t classes;       /* K, in [2, 255] */
    uint32_t reserved3;
    uint64_t offsets;       /* uint32_t[classes + 1]: OUT, exclusive prefix over the live samples */
    uint64_t class_sorts;   /* uint32_t[1]: incremented once when the permutation ran */
};

/* eagle_backend.h:814-824: permute every plane IN PLACE by a stable counting sort on
 * (live, class) over [0, *span) (dead last), then *count = *span = live; with
 * CLASSES_WITHIN_LIVE over [0, *count) by class only. perm moves, inv is rebuilt,
 * index_map is the identity over [0, live), offsets is written. */
eagle_backend_status eagle_backend_reorder_classes_device(struct eagle_backend_reorder_classes_desc* desc);

/* Residency classes of eagle_backend_pointer_residency (eagle_backend.h:833-839). */
#define EAGLE_BACKEND_RESIDENCY_HOST 0
#define EAGLE_BACKEND_RESIDENCY_DEVICE 1
#define EAGLE_BACKEND_RESIDENCY_MANAGED 2
#define EAGLE_BACKEND_RESIDENCY_MAPPED_HOST 3
#define EAGLE_BACKEND_RESIDENCY_PAGEABLE 4
#define EAGLE_BACKEND_RESIDENCY_OTHER_DEVICE 5
/* eagle_backend.h:847: classify ``ptr`` as seen from ``device`` (-1: the current one) */
eagle_backend_status eagle_backend_pointer_residency(int32_t device, uint64_t ptr, int32_t* cls);

/* The canonical sum of a compaction's survivors over several ranks with no host round
 * trip (this backend's addition; eagle folds per-rank partials of aligned shards in
 * rank order, eagle/exec/RankPartition.h:222-241, and has no ragged case). Rank r
 * holds ``kept`` = its c_r survivors in sample order. Two fixed-size blocks per rank
 * cross the ranks, each in one all-gather in rank order:
 *   the head block, 4096 float64: the rank's first min(c_r, 4095) survivors, then
 *     c_r as a uint32 in the low 32 bits of element 4095;
 *   the partial block, 2 * cap + 2 float64: the (hi, comp) partial of each leaf that
 *     starts in the rank's part, then their number as a uint32 in the low 32 bits of
 *     element 2 * cap (0xffffffff: a pass failed), element 2 * cap + 1 unused.
 * ragged_head writes rank r's head block (``count`` = c_r, uint32, on the device).
 * ragged_leaves reads ``blocks`` = every rank's head block ([world][4096]) and writes
 * rank r's partial block: every 4096-survivor leaf of the concatenation that STARTS in
 * rank r's part, its survivors past rank r's end taken from the later ranks' heads. */
eagle_backend_status eagle_backend_x_b200_ragged_head(uint64_t kept, uint64_t count, uint64_t block,
    uint64_t stream);
eagle_backend_status eagle_backend_x_b200_ragged_leaves(uint64_t kept, uint64_t blocks, int32_t rank,
    int32_t world, uint64_t partials, int64_t cap, uint64_t stream);
/* ragged_fold: every rank's partial block (``gathered`` = [world][2 * cap + 2],
 * all-gathered) through the canonical pairwise levels, in rank order, into ``out`` =
 * {hi, comp, value} (zeros for no survivors): the bits of the one-device
 * compact-then-sum of the concatenated shards. A rank whose leaves did not fit its
 * ``cap`` (ceil(shard samples / 4096) + 1 always fit) makes every rank's ``out`` NaN.
 * ``work`` holds 2 * ceil(world * cap / 512) + 2 doubles. */
eagle_backend_status eagle_backend_x_b200_ragged_fold(uint64_t gathered, int32_t world, int64_t cap,
    uint64_t work, uint64_t out, uint64_t stream);

/* compact-then-sum across ranks without writing the survivors (this backend's addition,
 * the fused form of ragged_head / ragged_leaves): x_b200_compact_sum cut where the ranks
 * exchange, with the same two blocks. Same desc and scratch as x_b200_compact_sum
 * (query there). _count: the keep bitmap, the tile counts and this rank's count (to
 * ``count``). _head (after _count): this rank's head block into ``block`` (4096
 * doubles); the caller all-gathers the head blocks into ``blocks`` ([world][4096],
 * rank order). _leaves (once per _count): from ``blocks`` on the device, the (hi, comp)
 * partial of every leaf of the concatenated survivors that starts and ends in this
 * rank, into ``partials`` (the partial block, 2 * cap + 2 doubles, cap >=
 * ceil(n / 4096) + 1) from index 0. _straddle: the leaf that starts here and runs into
 * the later ranks, from this rank's part and the later ranks' heads, after those
 * partials, and the block's leaf count. The partial blocks then go through
 * eagle_backend_x_b200_ragged_fold. */
eagle_backend_status eagle_backend_x_b200_compact_sum_count(struct eagle_backend_compact_desc* desc);
eagle_backend_status eagle_backend_x_b200_compact_sum_head(struct eagle_backend_compact_desc* desc,
    uint64_t values, uint64_t block);
eagle_backend_status eagle_backend_x_b200_compact_sum_leaves(struct eagle_backend_compact_desc* desc,
    uint64_t values, uint64_t blocks, int32_t rank, int32_t world, uint64_t partials, int64_t cap);
eagle_backend_status eagle_backend_x_b200_compact_sum_straddle(struct eagle_backend_compact_desc* desc,
    uint64_t blocks, int32_t rank, int32_t world, uint64_t partials, int64_t cap);

/* eagle_backend_x_b200_compact_wait_check: compact_device with its first tile withheld,
 * to exercise the bounded look-back wait (this backend's addition; eagle's multi-level
 * scan has no wait to bound, eagle/cuda/Scan.h:32-141). No CTA takes tile 0, so every
 * tile whose look-back reaches tile 0 polls its status word ``spin_limit`` times (in
 * [1, 2^22]; compact_device uses 2^22), gives up, sets the error word and goes on; the
 * last tile then writes a count of 0xffffffff, above any n, as compact_device does
 * after any wait that gave up. The map's contents are unspecified. Same desc and
 * caller scratch as compact_device; n must exceed one 32768-sample tile. */
eagle_backend_status eagle_backend_x_b200_compact_wait_check(struct eagle_backend_compact_desc* desc,
    uint32_t spin_limit);

/* eagle_backend_x_b200_compact_device_noalloc: compact_device for callers that
 * cannot allocate device memory (no counterpart in the reference: eagle's
 * compaction always takes caller scratch). Same desc, same outputs, same flags and
 * trigger; ``scratch`` must be 0 and no query is needed. Its working memory is a
 * fixed 64 KiB + 256 B array inside this library on every device that loads it,
 * enough for n <= 2^28 samples; a larger n returns UNSUPPORTED. It allocates
 * nothing: it enqueues one memset of that array and the compaction kernel. The
 * first call on a device looks the array's address up (cudaGetSymbolAddress) and
 * keeps it, so make that first call before any stream capture, and do not reset the
 * device (cudaDeviceReset) after it. Every call shares the one array:
 * calls that may overlap on the GPU (other streams, other threads) race and must
 * be serialised by the caller. */
eagle_backend_status eagle_backend_x_b200_compact_device_noalloc(struct eagle_backend_compact_desc* desc);

/* ---- canonical reduction (experimental; eagle_backend.h:896-906) -------------- */

/* The canonical fixed-order reduction of each column of the row-major (n, columns)
 * device plane ``in`` into ``out``: leaves of 256 slots x 16 strided samples, the
 * fixed in-leaf tree, level-by-level pairwise over the leaves. ``work_a == 0`` is
 * the query (writes work_elems). Every policy runs the ordered tree (bitwise
 * deterministic; the ordered result also meets the compensated contract). One
 * kernel per 65535 columns after a memset: enqueue only, capturable. */
eagle_backend_status eagle_backend_x_reduce_canonical(struct eagle_backend_reduce_desc* desc);

/* ---- this backend's additions (no counterpart entry in the seam) --------------- */

/* eagle_backend_x_b200_compact_gather: compact_device (same desc, query and
 * capturability) that also writes the kept samples' values, ``elem_bytes`` (4 or 8)
 * each from ``values``, in sample order to ``out_values[0, *count)``; ``index_map``
 * may be 0 (no map written). The compaction half of "compact the survivors, then
 * reduce them" (eagle: ActiveSet.compact, python/eagle/_active_set.py:482-525, then
 * a gather through the map) in one kernel. No reorder trigger. */
eagle_backend_status eagle_backend_x_b200_compact_gather(struct eagle_backend_compact_desc* desc, uint64_t values,
    uint64_t out_values, uint32_t elem_bytes);

/* eagle_backend_x_b200_reduce_counted: x_reduce_canonical (sums of F32 / F64 / I32 /
 * I64, one column, optional PAIR_OUT) of the first ``*count`` elements of ``in``
 * (``count`` a device uint32; ``desc->n`` the capacity, count is clipped to it),
 * read on the device: the reduction can follow compact_gather with no host read of
 * the count (eagle reads it back to size its reduce, python/eagle/_graph_reduce.py
 * :204-222). Same bits as x_reduce_canonical over that many elements; 0 elements
 * give 0. Query with work_a == 0. One kernel after a memset; capturable. */
eagle_backend_status eagle_backend_x_b200_reduce_counted(struct eagle_backend_reduce_desc* desc, uint64_t count);

/* eagle_backend_x_b200_reduce_fixed: x_reduce_canonical of float64 sums on eagle's
 * fixed-point leaf (eagle/reduce/canonical.h:153-302): the same tree over 128-bit
 * fixed-point partials (v * 2^u, the unit 106 bits below the largest term; IEEE
 * specials as sticky flags; one rounding at the end), the path eagle takes -- and
 * x_reduce_canonical takes by itself -- on a device whose FP32:FP64 throughput ratio
 * is 8 or worse (canonical.h:304-313). Offered here on any device so that its bits
 * can be had and checked on B200 too. dtype F64, op SUM, any policy, columns and
 * comp_in as x_reduce_canonical; PAIR_OUT returns UNSUPPORTED. Query with
 * work_a == 0. One kernel per 65535 columns after a memset; capturable. */
eagle_backend_status eagle_backend_x_b200_reduce_fixed(struct eagle_backend_reduce_desc* desc);

/* eagle_backend_x_b200_compact_sum: the canonical ordered sum of the float64
 * ``values`` the mask keeps, in sample order -- the bits of compact_gather followed
 * by reduce_counted -- without writing the kept values anywhere: the mask becomes a
 * keep bitmap with per-tile counts, a scan of the counts gives the sample where every
 * 4096-survivor leaf begins, and each leaf is summed straight from ``values``. Writes
 * ``*count`` (the survivors) and ``out[0]`` (the sum), or with ``flags`` =
 * EAGLE_BACKEND_REDUCE_PAIR_OUT ``out[0..1]`` = (hi, comp). Same desc as
 * compact_device: ``index_map`` and the trigger fields must be 0 (no map is
 * written), MASK_IS_DROP honoured, ``scratch == 0`` is the query (scratch_bytes; the
 * size depends on the device's SM count), scratch 256-byte aligned, n <= 2^31-1. A
 * leaf whose bitmap and start disagree (the mask changed under the call) stores
 * count 0xffffffff and a NaN sum. One memset and four kernels, no wait on another
 * CTA: enqueue only, capturable. */
eagle_backend_status eagle_backend_x_b200_compact_sum(struct eagle_backend_compact_desc* desc, uint64_t values,
    uint64_t out, uint32_t flags);

/* No counterpart in the reference: every leaf's (hi, comp) partial of a float64 sum
 * of ``n`` elements into ``out[2 * leaves]`` (the last leaf over the remainder) --
 * the leaves of the canonical tree (canonical.h:340-353), so that leaves whose
 * elements live on several ranks (a compaction's ragged survivors) can be formed
 * where their elements meet and then joined by x_b200_combine_partials. */
eagle_backend_status eagle_backend_x_b200_leaf_partials(uint64_t in, int64_t n, uint64_t out, uint64_t stream);

/* eagle_backend_x_b200_combine_partials: combine ``m`` float64 (hi, comp) partials
 * ``hc[2m]`` (chunk roots in chunk order, e.g. one per rank; each chunk
 * leafSize * 2^q samples) by the canonical pairwise levels into ``out[3]`` = {hi,
 * comp, value}: the bits of the reduction over the concatenated chunks
 * (eagle/reduce/canonical.h:30-32, :424-439, the rank-order fold of
 * eagle/exec/RankPartition.h:230-241). ``work`` holds 2 * ceil(m / 512) doubles
 * (unused for m == 1). One single-CTA kernel; enqueue only. */
eagle_backend_status eagle_backend_x_b200_combine_partials(uint64_t hc, int64_t m, uint64_t work, uint64_t out,
    uint64_t stream);

/* eagle_backend_x_b200_entry: the CUfunction (as uint64) of one of this backend's
 * built-in step kernels by name, for run_device / launch_raw. The kernels take the
 * hawk argument ABI: role arguments packed as eagle's registry packs them
 * (plugin/plugin_registry/registry.h:605-710: a 32-byte handle per per-sample,
 * mutable, terminated and lookup plane, float64 uniforms by value), then
 * ``int64 base, count, nSamples`` (eagle/exec/DeviceKernel.h:47-84), then the
 * fast-entry tails of python/eagle/_plan_binding.py:455-460 (``_persist``) and
 * :582-591 (``_range``). Names: "oscillator", "oscillator_range", "oscillator_persist"
 * (t_end a Param) and "oscillator_spread", "..._range", "..._persist" (t_end per
 * sample); a "_fma" suffix selects the contracted multiply-adds. */
eagle_backend_status eagle_backend_x_b200_entry(const char* name, int32_t device, uint64_t* function);

/* The until-done engine (this backend's addition; it stands in for the loop that
 * python/eagle/_until_done.py:528-1845 builds from seam calls). One engine runs one
 * model over n samples resident on one device. */
#define EAGLE_B200_MODEL_OSCILLATOR 0u        /* README.md:89-97, t_end a Param */
#define EAGLE_B200_MODEL_OSCILLATOR_SPREAD 1u /* the same body, t_end per sample */
#define EAGLE_B200_MODEL_GAMBLER 2u           /* +-1 walk absorbed at 0 and 100, Philox-4x32-10 steps */
#define EAGLE_B200_MODEL_LORENZ 3u            /* Lorenz-63 under adaptive RKF7(8); a step is one attempt */

#define EAGLE_B200_MODE_BAND 0u    /* one CUDA graph: WHILE { fused step + compaction + policy } */
#define EAGLE_B200_MODE_PERSIST 1u /* one persistent launch: lanes claim samples off a counter */
#define EAGLE_B200_MODE_FUSED 2u   /* one launch, one lane per sample, the whole budget */
#define EAGLE_B200_MODE_BAND_EAGER 3u /* the band passes launched from the host, one condition read per pass */

#define EAGLE_B200_FLAG_FMA 1u /* contract x0 + dt*v0 and v0 - c*x0 into fused multiply-adds */
/* persist oscillator: claim samples in index order. By default the engine first orders each
 * run of 32768 samples by their stop steps, estimated as (t_end - t) / dt, longest first, and
 * the lanes claim them in that order (a warp's lanes then run samples of like length); the
 * planes, mask and report are the same bits either way. The order holds 4 bytes per sample
 * of device memory. */
#define EAGLE_B200_FLAG_INDEX_ORDER 2u

struct eagle_b200_engine_desc {
    uint32_t struct_size;
    uint32_t flags;      /* EAGLE_B200_FLAG_* */
    int32_t device;      /* -1: the device owning the planes */
    uint32_t model;      /* EAGLE_B200_MODEL_* */
    uint32_t mode;       /* EAGLE_B200_MODE_* */
    uint32_t reserved0;
    int64_t n;           /* samples, 0 <= n <= 2^31 - 1 */
    int64_t max_steps;   /* steps a sample may take per run, >= 0 */
    uint64_t planes[8];  /* device addresses of the model's planes, in the model's order */
    double uniforms[4];  /* the model's Params, in the model's order */
    uint64_t terminated; /* u8[n] mask: a set byte is a finished sample */
    int64_t k_first;     /* band: steps of the first launch (0: 16) */
    int64_t k_min;       /* band: fewest steps per launch but the last (0: 8) */
    int64_t k_max;       /* band: most steps per launch (0: 4096) */
    uint32_t chunk;      /* persist: steps between claims, a power of two (0: the oscillator 4096
                          * claimed longest first, 512 in index order; GAMBLER 256; LORENZ 8) */
    uint32_t block;      /* threads per block (0: 256) */
    double overhead_steps; /* band: a launch's fixed cost in sample-steps (0: built-in) */
    double interval_steps; /* band: a launch's per-sample memory cost in steps (0: built-in) */
    int64_t iuniforms[4];  /* the model's integer Params, in the model's order */
    double uniforms_ext[4]; /* the model's float Params past the first four */
    uint32_t ctas_per_sm;   /* persist: resident CTAs per SM (0: as many as fit); fewer leave room
                             * for runs on other streams to overlap this run's tail */
    uint32_t reserved1;
};

/* What one run did (python/eagle/_until_done.py:120-171, RunReport). */
struct eagle_b200_report {
    uint32_t struct_size;
    uint32_t done;        /* finished == n */
    int64_t n;
    int64_t finished;     /* samples whose mask is set when the run ends */
    int64_t steps;        /* the longest sample's steps in this run (exact) */
    int64_t launches;     /* loop iterations (band) or 1 */
    int64_t compactions;  /* compactions run (band) */
    uint64_t step_sum;    /* steps executed by all samples in this run */
    uint32_t error;       /* device error word: 0 = none (bit 0: a look-back wait gave up,
                           * bit 1: the band loop was stopped by its pass guard) */
    uint32_t mode;
    uint32_t report_bytes; /* bytes the report read moved device -> host */
    uint32_t reserved0;
};

/* The models' plane orders: OSCILLATOR planes = {omega, x, v, t}, uniforms = {t_end,
 * dt}; OSCILLATOR_SPREAD planes = {omega, t_end, x, v, t}, uniforms = {dt};
 * GAMBLER planes = {pos (int32), time (int64)}, iuniforms = {seed, id_base};
 * LORENZ planes = {rho, x, y, z, t, h, n_acc (uint32), n_rej (uint32)}, uniforms =
 * {sigma, beta, t_final, rtol}, uniforms_ext = {atol}. GAMBLER and LORENZ run under
 * the persist and fused modes. */
typedef struct eagle_b200_engine_s* eagle_b200_engine;

/* Allocate the engine's device state (compacted state, look-back words, cells) on
 * its device and, for the band mode, build its graph. Allocates: call outside any
 * stream capture. */
eagle_backend_status eagle_backend_x_b200_engine_create(const struct eagle_b200_engine_desc* desc,
    eagle_b200_engine* out);
/* Enqueue one run on ``stream`` (continuing from the current mask and state);
 * no host synchronisation. */
eagle_backend_status eagle_backend_x_b200_engine_launch(eagle_b200_engine h, uint64_t stream);
/* Wait for ``stream`` and read the last run's report (one device-to-host copy). */
eagle_backend_status eagle_backend_x_b200_engine_report(eagle_b200_engine h, uint64_t stream,
    struct eagle_b200_report* report);
/* The report in two halves, so that many engines' reports cost one host wait:
 * report_enqueue puts the device-to-host copy of the run's counters on ``stream``
 * (no wait); report_read fills ``report`` from that copy and must follow a wait
 * for the stream (cudaStreamSynchronize, an event, ...) that covers the copy. */
eagle_backend_status eagle_backend_x_b200_engine_report_enqueue(eagle_b200_engine h, uint64_t stream);
eagle_backend_status eagle_backend_x_b200_engine_report_read(eagle_b200_engine h, struct eagle_b200_report* report);
/* launch + report. */
eagle_backend_status eagle_backend_x_b200_engine_run(eagle_b200_engine h, uint64_t stream,
    struct eagle_b200_report* report);
void eagle_backend_x_b200_engine_release(eagle_b200_engine h);
/* Timing of the engine's main kernel (this backend's addition, for measurement; eagle
 * times whole launches from Python, python/eagle/_until_done.py:1322-1460): arm CUDA
 * events recorded on the launch stream just before and just after the main kernel
 * (the persistent or fused step entry; the band graph as a whole) of each of the
 * next ``launches`` launches, in [0, 65536]; 0 disarms. Re-arming drops earlier
 * times. Creates events: call outside any stream capture. */
eagle_backend_status eagle_backend_x_b200_engine_time_kernel(eagle_b200_engine h, int32_t launches);
/* Wait for the timed launches' events and write the first min(cap, timed) kernel
 * times in milliseconds to ``ms``; ``*count`` = launches timed since arming. */
eagle_backend_status eagle_backend_x_b200_engine_kernel_ms(eagle_b200_engine h, float* ms, int32_t cap,
    int32_t* count);

/* The FP64 issue probe (this backend's addition, for measurement; no counterpart in
 * eagle): times a kernel of fused double-precision multiply-adds on ``device`` (-1:
 * the current one) and writes the best rate of five launches, in lane multiply-adds
 * per second. ``kind`` 0..3: 1, 2, 4 or 8 independent chains per lane, c = fma(c, a,
 * b) with a and b arguments; 4..6: the oscillator's step on 1, 2 or 3 samples per
 * lane, x' = fma(dt, v, x) and v' = fma(-c, x, v), whose two multiply-adds need both
 * results of the step before. ``ctas_per_sm``: resident CTAs of 256 threads per SM (0:
 * as many as fit). Synchronises ``stream`` and allocates stream-ordered memory: not
 * for use inside a capture. */
eagle_backend_status eagle_backend_x_b200_probe_fp64(int32_t device, uint32_t kind, uint32_t ctas_per_sm,
    uint64_t stream, double* fma_per_s);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* EAGLE_B200_H */
