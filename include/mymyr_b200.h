/* mymyr_b200: the B200 (sm_100a) device path of the mymyr lifted planner, behind a C ABI.
 *
 * The path: batched lifted successor generation over packed ground-atom bitset states, 64-bit state hashing with an
 * open-addressing device hash set that deduplicates each breadth-first layer, and the batched RL environment step.
 * Every entry point takes plain pointers and sizes; device buffers are caller-owned (destination passing) unless an
 * object (b2_brfs) owns them. No C++ exception crosses this boundary: every call returns a b2_status and
 * b2_last_error() describes the last failure of the calling thread.
 *
 * State rows follow the reference's word contract (include/mymyr/core/bitset.hpp:1-10 and
 * include/mymyr/state/state.hpp:1-13 in maichmueller/mymyr): little-endian u64 words, fluent slot i is bit i & 63
 * of word i >> 6, slot = the atom's canonical id (TaskOptions::Atoms::Dense, include/mymyr/task/atom_index.hpp:9-20).
 * Hashes are the reference's hash::state over the trimmed words (include/mymyr/core/hash.hpp:38-60), bit for bit.
 *
 * Streams are passed as `void*` (a cudaStream_t; NULL is the legacy default stream). Every device pointer must be
 * memory of the context's device.
 */
#ifndef MYMYR_B200_H
#define MYMYR_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes. The C++ shim maps them onto the reference's exceptions: INVALID_ARGUMENT and UNSUPPORTED ->
 * std::invalid_argument, CAPACITY -> std::length_error, PARSE -> std::runtime_error, CUDA and DEVICE -> CudaError
 * (include/mymyr/cuda/runtime.hpp:31-45). */
typedef enum b2_status {
    B2_OK = 0,
    B2_INVALID_ARGUMENT = 1, /* malformed call: null or mismatched buffers, out-of-range ids */
    B2_UNSUPPORTED = 2,      /* a task feature the device path does not run (numeric fluents, axioms, ...) */
    B2_CAPACITY = 3,         /* an output or arena capacity is too small; the call can be repeated with more */
    B2_CUDA_ERROR = 4,       /* a CUDA runtime call failed */
    B2_DEVICE_FAULT = 5,     /* a kernel reported a sticky status bit (probe limit, bounded wait ran out) */
    B2_PARSE_ERROR = 6       /* the task text is malformed */
} b2_status;

typedef struct b2_ctx b2_ctx;
typedef struct b2_task b2_task;
typedef struct b2_brfs b2_brfs;
typedef struct b2_env b2_env;

/* Copies the calling thread's last error message (NUL-terminated, truncated to cap) and returns its full length.
 * Replaces the what() of the reference's exceptions. */
size_t b2_last_error(char* buf, size_t cap);

/* Library version string. */
const char* b2_version(void);

/* ------------------------------------------------------------------------------------------------ context
 * One context per device: its stream-ordered scratch pool, status words and the device properties.
 * Replaces mymyr::cuda::DeviceContext::create (include/mymyr/cuda/runtime.hpp:148). */
b2_status b2_ctx_create(int device, b2_ctx** out);
void b2_ctx_destroy(b2_ctx* ctx);

/* ------------------------------------------------------------------------------------------------ task
 * A normalized lifted STRIPS task as flat pools: the fields of formalism::TaskData
 * (include/mymyr/formalism/task_data.hpp:24-33, 317-370) that the path reads. Terms: >= 0 a parameter index of the
 * enclosing schema, < 0 object o as -(o + 1). Atom records are [pred, args...] with the predicate's arity. */
typedef struct b2_literal {
    uint32_t pred;
    uint32_t positive;
    uint32_t term_begin; /* into terms */
    uint32_t term_count; /* the predicate's arity */
} b2_literal;

typedef struct b2_schema_desc {
    uint32_t arity;
    uint32_t pre_begin, pre_count; /* precondition literals, into literals */
    uint32_t eff_begin, eff_count; /* unconditional effect literals (positive: add, negative: delete) */
    const char* name;              /* optional (may be NULL) */
} b2_schema_desc;

enum { B2_PRED_STATIC = 0, B2_PRED_FLUENT = 1, B2_PRED_DERIVED = 2 };

typedef struct b2_task_desc {
    uint32_t num_objects;
    uint32_t num_predicates;
    const uint8_t* pred_kind;   /* B2_PRED_* per predicate */
    const uint32_t* pred_arity; /* per predicate */
    const int32_t* terms;
    uint32_t num_terms;
    const b2_literal* literals;
    uint32_t num_literals;
    const b2_schema_desc* schemas;
    uint32_t num_schemas;
    const uint32_t* static_init; /* atom records */
    uint64_t static_init_words;
    const uint32_t* fluent_init; /* atom records */
    uint64_t fluent_init_words;
    uint32_t goal_begin, goal_count; /* ground goal literals, into literals */
    uint32_t unsupported;            /* nonzero: the source had features the device path does not run */
} b2_task_desc;

/* Reads the reference's normalized task text format (include/mymyr/formalism/text_format.hpp:1-23; the plain lifted
 * variant "O P SI FI G A") into a library-owned description. Numeric sections, axioms (X), collapsed parameters (C)
 * and conditional effects parse into desc->unsupported != 0, which b2_task_create refuses. */
b2_status b2_task_desc_read_text(const char* text, size_t len, b2_task_desc** out);
void b2_task_desc_free(b2_task_desc* desc);

/* Compiles the description (the typed-dense canonical atom layout of the reference's compile step,
 * src/mymyr/task/compile.cpp:1103-1180, with slot = canonical id) and uploads the matcher tables to the context's
 * device. Replaces Task::create + rl::device_arrays (include/mymyr/rl/task_arrays.hpp:247-256) on this path.
 * ctx may be NULL: the task is then compiled on the host only (layout, initial state, slot records) and every
 * device entry point refuses it with B2_INVALID_ARGUMENT. */
b2_status b2_task_create(b2_ctx* ctx, const b2_task_desc* desc, b2_task** out);
void b2_task_destroy(b2_task* task);

/* How the kernels match schema preconditions. COMPILED (the default): the task's matchers are generated as CUDA with
 * every layout constant folded in and compiled for sm_100a at task creation (NVRTC, cached per process by program);
 * INTERPRETED: generic kernels walk the task's matcher tables. Both enumerate the same bindings in the same order. */
enum { B2_MATCHER_AUTO = 0, B2_MATCHER_INTERPRETED = 1, B2_MATCHER_COMPILED = 2 };

typedef struct b2_task_options {
    int32_t matcher; /* B2_MATCHER_* */
} b2_task_options;

/* b2_task_create with options (NULL: the defaults). */
b2_status b2_task_create_ex(b2_ctx* ctx, const b2_task_desc* desc, const b2_task_options* options, b2_task** out);

/* Compiles the task's kernels for sm_100a into the process cache without a device (a host-only task works). The
 * generated source is copied into src (NUL-terminated, truncated to src_cap; src may be NULL) and its full length
 * returned in *src_len (may be NULL). */
b2_status b2_task_compile(const b2_task* task, char* src, size_t src_cap, size_t* src_len);

typedef struct b2_task_info {
    uint32_t words;        /* Task::words(): u64 words of a state row */
    uint32_t fluent_slots; /* AtomIndex::fluent_slots() */
    uint32_t num_schemas;
    uint32_t num_objects;
    uint32_t label_width;  /* largest schema arity (rl::max_label_width) */
    uint32_t object_words; /* words of an object bitset */
} b2_task_info;
b2_status b2_task_info_get(const b2_task* task, b2_task_info* out);

/* The initial state (Task::initial_state), zero-padded to `words` words, into host memory. */
b2_status b2_task_initial_state(const b2_task* task, uint64_t* row, uint32_t words);
/* The predicate and objects of fluent slot `slot` (AtomIndex::record): pred_args[0] = pred, then its arity objects. */
b2_status b2_task_slot_atom(const b2_task* task, uint32_t slot, uint32_t* pred_args, uint32_t cap);

/* ------------------------------------------------------------------------------------------------ hashing
 * hash::state of n device rows of `words` words into out[n] (device). Replaces hash_rows
 * (python/src/module.cpp:187) for classical rows (numeric_words = 0). */
b2_status b2_hash_rows(b2_ctx* ctx, const uint64_t* rows, uint64_t n, uint32_t words, uint64_t* out, void* stream);
/* hash_rows with numeric words: each row is [words - numeric_words atom words | numeric_words numeric words], hashed
 * as hash::state (include/mymyr/core/hash.hpp:55-60): the trimmed atom words seeded by hash::words of the numeric
 * words. numeric_words = 0 is b2_hash_rows. */
b2_status b2_hash_rows_numeric(b2_ctx* ctx, const uint64_t* rows, uint64_t n, uint32_t words, uint32_t numeric_words,
                               uint64_t* out, void* stream);

/* ------------------------------------------------------------------------------------------------ batched expand
 * rl::expand (include/mymyr/rl/expand.hpp:137-147) on the device: the successors of n states in canonical order
 * (schema, then binding), as CSR. All arrays are device memory; a NULL array is not written. Rows beyond `capacity`
 * are counted, not written (generated > capacity is the overflow, B2_CAPACITY). */
typedef struct b2_expansion {
    uint64_t capacity;
    uint32_t words;       /* words per succ row */
    uint32_t label_width; /* columns of binding (>= label_width of the task when binding is set) */
    uint64_t* succ;       /* [capacity, words] */
    int32_t* parent;      /* [capacity] */
    int32_t* schema;      /* [capacity] */
    int32_t* binding;     /* [capacity, label_width]; -1 past the schema's arity */
    int32_t* offsets;     /* [rows + 1] */
    uint64_t* succ_hash;  /* [capacity]: State::hash() of the successor */
    uint64_t generated;   /* out: successors of the whole batch */
} b2_expansion;
b2_status b2_expand(b2_task* task, const uint64_t* states, uint64_t rows, uint32_t words, int witness_pruning,
                    b2_expansion* out, void* stream);

/* b2_expand for callers that cannot allocate device memory while they run: processes that reserve the GPU's memory up
 * front through their own allocator (a framework's caching allocator, a fixed per-process budget) and forbid other
 * allocations, and latency-bound callers that cannot take the device-wide synchronization of cudaMalloc/cudaFree. It
 * has no counterpart in the reference. Same arguments, results and errors as b2_expand; it calls no cudaMalloc,
 * cudaFree or other allocating routine. Its scratch is a fixed array in the library's device memory (about 3 MB, held
 * by every GPU that loads the library until the process exits), so a call takes at most 2^18 (state, schema) segments
 * (rows x schemas) and refuses larger batches with B2_CAPACITY. Whatever it needs is set up before its first call:
 * b2_ctx_create loads the array and the call's kernels on the device and looks up the array's device address (once
 * per context), b2_task_create loads the task's compiled kernels. All calls on a device share the one array, which
 * keeps the last call's contents (each call zeroes what must start at zero); two calls running on the GPU at the same
 * time would race on it, so the library runs them one at a time: a process-wide lock, and each call returns only
 * after its stream has finished the work. */
b2_status b2_expand_noalloc(b2_task* task, const uint64_t* states, uint64_t rows, uint32_t words, int witness_pruning,
                            b2_expansion* out, void* stream);

/* ------------------------------------------------------------------------------------------------ communicators
 * Multi-GPU searches run one process (or host thread) per GPU. Their ranks share an NCCL communicator for the
 * reductions of each layer and map each other's receive buffers (CUDA IPC) for the exchange of successors. The
 * reference has no multi-GPU layer; these have no counterpart in it. NCCL (libnccl.so.2) is loaded on first use;
 * in a process that already loaded it (PyTorch) that copy is used. */
typedef struct b2_comm b2_comm;
typedef struct b2_comm_id {
    char bytes[128]; /* an ncclUniqueId: made once (b2_comm_id_new) and handed to every rank */
} b2_comm_id;
b2_status b2_comm_id_new(b2_comm_id* out);
/* Collective: every rank of `world` calls it with the same id and its own rank, on its own GPU's context. */
b2_status b2_comm_create(b2_ctx* ctx, const b2_comm_id* id, uint32_t rank, uint32_t world, b2_comm** out);
/* Seconds a rank waits for the others' part of a collective before it aborts the communicator and fails the call
 * with B2_CUDA_ERROR (default 600): a rank that stopped taking part ends the others' searches instead of hanging them. */
b2_status b2_comm_set_timeout(b2_comm* comm, double seconds);
/* Releases the communicator. Collective: every rank destroys it, after the last search over it has ended on every
 * rank (NCCL's teardown waits for the other ranks). */
void b2_comm_destroy(b2_comm* comm);

/* ------------------------------------------------------------------------------------------------ BrFS
 * The layer-synchronous breadth-first search of cuda::DeviceBrfs (include/mymyr/cuda/brfs.hpp:96-123) and mymyr::brfs
 * (include/mymyr/search/brfs.hpp:140): same states, ids, per-layer counts and fingerprint as the reference CPU BrFS
 * with deterministic ids. The state space stays on the device until b2_brfs_destroy.
 *
 * With a communicator the search is sharded over its ranks: every state lives on the rank its hash::state selects
 * (owner = high 32 bits of the hash x ranks >> 32), each rank expands the states it owns, and the successors go to
 * their owners. Every rank calls b2_brfs_create and b2_brfs_run together and gets the same result; the ids, layer
 * counts and fingerprint are those of the one-GPU search. A rank reads its own states with b2_brfs_local. */
typedef struct b2_brfs_options {
    int32_t witness_pruning;  /* default 1 */
    int32_t stop_at_goal;     /* default 1 */
    int32_t fingerprint;      /* default 0 */
    uint32_t max_depth;       /* expand states of depth < max_depth (0xFFFFFFFF: no limit) */
    uint64_t max_states;      /* 0xFFFF...: no limit */
    uint64_t expected_states; /* pre-sizes the table and arenas (0: grow as needed) */
    int32_t timings;          /* per-phase device times in b2_brfs_result */
    int32_t world_rank;       /* multi-GPU: this rank (0 for one GPU; the communicator's rank when `comm` is set) */
    int32_t world_size;       /* multi-GPU: ranks sharing the frontier by state-hash owner (1: one GPU) */
    void* stream;             /* the stream the search runs on (NULL: a stream of its own) */
    b2_comm* comm;            /* multi-GPU: the ranks' communicator (NULL: one GPU) */
    uint64_t max_exchange_records; /* multi-GPU: the most successor records a rank takes in per layer (0: as many
                                    * as the layer needs; the receive buffers grow to them). A layer that needs more
                                    * fails on every rank with B2_CAPACITY: records past a buffer are never written */
    uint64_t shard_from_states;    /* multi-GPU: every rank runs the layers alone, the same search with no exchange,
                                    * until a layer's frontier holds at least this many states; the ranks then keep
                                    * the states they own and shard the rest of the search (0: 2^20; 1: shard from
                                    * the root). The result does not depend on it */
} b2_brfs_options;

void b2_brfs_options_default(b2_brfs_options* o);

enum { B2_SEARCH_SOLVED = 0, B2_SEARCH_EXHAUSTED = 1, B2_SEARCH_OUT_OF_STATES = 2, B2_SEARCH_UNSOLVABLE = 3 };

typedef struct b2_brfs_result {
    uint32_t status;           /* B2_SEARCH_* */
    uint32_t layers;           /* layers expanded */
    uint64_t states;           /* stored states */
    uint64_t expanded;
    uint64_t generated;
    uint64_t num_goal_states;
    int32_t exhausted;
    int32_t solved;
    uint64_t goal_id;          /* the first goal state expanded (solved only) */
    uint64_t fingerprint;      /* xor of brfs_fingerprint_term(id, canonical hash) (options.fingerprint) */
    double search_s;           /* wall time of the search */
    double count_ms;           /* device time of the count passes (goal test + successor counts + offsets scan) */
    double gen_ms;             /* device time of the expansion passes (regenerate, hash, insert; options.timings) */
    double dedup_ms;           /* device time of id assignment (scan of the layer's winners; options.timings) */
    uint64_t kernel_launches;  /* kernels this search launched */
    uint64_t* layer_counts;    /* in: caller buffer [layer_capacity, 3] (host) or NULL; out: {expanded, generated, new} */
    uint32_t layer_capacity;
    uint32_t table_log2;       /* out: log2 of the hash-set slots at the end */
    uint32_t rehashes;         /* out: table growths */
    uint32_t words;
    uint64_t local_states;     /* out: states this rank stores (all of them on one GPU) */
    uint64_t exchanged;        /* out: successors this rank received from other ranks (sharded search) */
    double exchange_ms;        /* out: sharded search: device time of the successor exchange (per-owner counts,
                                  push, barrier; options.timings), part of gen_ms */
    double wait_ms;            /* out: host time spent waiting for the device's per-layer results (of search_s) */
} b2_brfs_result;

b2_status b2_brfs_create(b2_task* task, const b2_brfs_options* options, b2_brfs** out);
b2_status b2_brfs_run(b2_brfs* search, b2_brfs_result* result);
/* State rows [first, first + count) in id order, `words` words each, into host memory. */
b2_status b2_brfs_states(b2_brfs* search, uint64_t first, uint64_t count, uint64_t* rows, uint32_t words);
/* Node records {parent id, successor index} of states [first, first + count) (the root's parent is 0xFFFFFFFF). */
b2_status b2_brfs_nodes(b2_brfs* search, uint64_t first, uint64_t count, uint32_t* parent, uint32_t* index);
/* hash::state of every stored state, in id order, into host memory (the visited-state hash set). */
b2_status b2_brfs_state_hashes(b2_brfs* search, uint64_t first, uint64_t count, uint64_t* hashes);
/* The states this rank stores (all of them on one GPU), in id order: their count, and for local states
 * [first, first + count) their ids, rows (`words` words each), hashes and node records, into host memory (NULL arrays
 * are skipped). The states, nodes and state_hashes calls above serve one-GPU searches only. No counterpart in the
 * reference (it has no sharded search). */
b2_status b2_brfs_local_count(b2_brfs* search, uint64_t* count);
b2_status b2_brfs_local(b2_brfs* search, uint64_t first, uint64_t count, uint64_t* ids, uint64_t* rows, uint32_t words,
                        uint64_t* hashes, uint32_t* parent, uint32_t* index);
void b2_brfs_destroy(b2_brfs* search);

/* ------------------------------------------------------------------------------------------------ h^max
 * The delete-relaxation heuristic h^max with unit costs (heuristics::Kind::Max; RelaxedTask grounding,
 * include/mymyr/heuristics/relaxed_task.hpp:1-22; evaluation src/mymyr/heuristics/heuristics.cpp:185-420), evaluated on
 * the device like cuda::DeviceHeuristic::evaluate (include/mymyr/cuda/heuristics.hpp:115). Creating it grounds the
 * relaxation on the host from the task's initial state; tasks with negative preconditions or goals are refused
 * (B2_UNSUPPORTED). A host-only task grounds (b2_heuristic_info_get) but cannot evaluate. */
typedef struct b2_heuristic b2_heuristic;
enum { B2_HEURISTIC_MAX = 2 }; /* heuristics::Kind::Max */
#define B2_DEAD_END 0xFFFFFFFFu /* h of a dead end (DeviceHeuristic::k_dead_end) */

typedef struct b2_heuristic_info {
    uint32_t props;            /* propositions: the task's fluent slots */
    uint32_t ops;              /* relaxed operators kept (those that add an atom outside their preconditions) */
    uint64_t reached_atoms;    /* GroundingStats::reached_atoms: atoms of the delete-free fixpoint */
    uint64_t ground_actions;   /* GroundingStats::ground_actions */
    uint32_t goal_atoms;
    uint32_t goal_unreachable; /* a goal atom is never reached: every state is a dead end */
} b2_heuristic_info;

b2_status b2_heuristic_create(b2_task* task, int32_t kind, b2_heuristic** out);
b2_status b2_heuristic_info_get(const b2_heuristic* h, b2_heuristic_info* out);
/* h of the n device rows rows + i * stride (`words` = the task's words) into out[0, n) (device u32, B2_DEAD_END for
 * dead ends), on `stream`. */
b2_status b2_heuristic_evaluate(b2_heuristic* h, const uint64_t* rows, uint64_t stride, uint32_t words, uint64_t n,
                                uint32_t* out, void* stream);
void b2_heuristic_destroy(b2_heuristic* h);

/* ------------------------------------------------------------------------------------------------ A*
 * Eager A* with h^max and unit costs (search::astar_eager, include/mymyr/search/best_first.hpp:9-15, 191;
 * cuda::astar, include/mymyr/cuda/astar.hpp:110): the optimal plan cost of the reference. Each device step expands
 * every open state of the lowest f at once (the reference's DeviceBestFirstOptions::single_bucket = false), so
 * `expanded` and `generated` count the states of the final f layer that a one-at-a-time search leaves unexpanded. */
typedef struct b2_astar b2_astar;

typedef struct b2_astar_options {
    uint64_t max_expansions;   /* 0: no limit (the search stops with B2_SEARCH_OUT_OF_STATES past it) */
    uint64_t expected_states;  /* pre-sizes the state arena and table (0: grow) */
    int32_t witness_pruning;   /* default 0, as the reference's A* */
    int32_t timings;           /* per-phase device times */
    void* stream;              /* NULL: a stream of its own */
    b2_heuristic* heuristic;   /* an h^max of the same task to share (NULL: the search grounds its own) */
    uint64_t chunk_candidates; /* successors staged at once: an f layer with more is expanded in chunks (bounded
                                  memory; 0: 2^26; at least 2^16; one GPU) */
    b2_comm* comm;             /* multi-GPU: states partitioned by state-hash owner over the communicator's ranks, every
                                  rank calls create and run together and gets the same result (no plan; no counterpart
                                  in the reference) */
} b2_astar_options;

void b2_astar_options_default(b2_astar_options* o);

typedef struct b2_astar_result {
    uint32_t status;           /* B2_SEARCH_SOLVED, _EXHAUSTED (no plan), _UNSOLVABLE (dead-end or goal-false start),
                                  _OUT_OF_STATES (max_expansions) */
    uint32_t waves;            /* device steps (batches of equal f) */
    double cost;               /* g of the goal state (solved) */
    uint64_t expanded, generated, states, evaluations, dead_ends;
    double initial_h;          /* -1: a dead end */
    uint32_t f_layers;         /* f values expanded */
    uint32_t plan_length;
    double search_s, count_ms, expand_ms, insert_ms, eval_ms;
    uint64_t kernel_launches;
    uint64_t relaxed_ops, relaxed_atoms;
} b2_astar_result;

/* The task (and a shared heuristic) must outlive the search object. */
b2_status b2_astar_create(b2_task* task, const b2_astar_options* options, b2_astar** out);
b2_status b2_astar_run(b2_astar* search, b2_astar_result* result);
/* The plan as its states' transitions, root first: step i leaves state parent[i] (a state index of the search) by its
 * index[i]-th successor in canonical order; *len = the plan length (steps are written when cap >= *len). */
b2_status b2_astar_plan(b2_astar* search, uint32_t* parent, uint32_t* index, uint32_t cap, uint32_t* len);
void b2_astar_destroy(b2_astar* search);

/* ------------------------------------------------------------------------------------------------ env step
 * The batched environment of rl::HostEnv / cuda::DeviceEnv (include/mymyr/rl/env.hpp:214-260,
 * include/mymyr/cuda/env.hpp:125-198) over one task, Index action space, random policy or given actions. */
typedef struct b2_env_config {
    uint64_t seed;
    uint32_t max_steps;       /* 0: never truncate */
    float step_reward;
    float goal_reward;        /* default 1 */
    float dead_end_reward;
    int32_t dead_end_none;    /* 1: DeadEnd::None */
    int32_t dead_end_terminal;/* default 1 */
    int32_t autoreset;        /* default 1 (SAME_STEP) */
    int32_t witness_pruning;  /* default 0 */
} b2_env_config;

void b2_env_config_default(b2_env_config* c);

typedef struct b2_env_batch {
    uint64_t* states;   /* [rows, words] device */
    uint64_t rows;
    uint32_t words;
    int32_t* steps;     /* [rows] */
    uint64_t* draws;    /* [rows] RNG draw counters */
    uint8_t* at_goal;   /* [rows] required */
    uint32_t* counts;   /* [rows, num_schemas] per-schema successor counts of the current states (required; written
                           by reset and step) */
    uint64_t first_env; /* the RNG stream of row 0 */
} b2_env_batch;

typedef struct b2_step_out {
    float* reward;
    uint8_t* terminated;
    uint8_t* truncated;
    int32_t* count;
    uint64_t* final_states; /* [rows, words] */
    int32_t* schema;
    int32_t* binding;       /* [rows, label_width] */
    uint32_t label_width;
    uint8_t* invalid;
    uint8_t* goal;
} b2_step_out;

b2_status b2_env_create(b2_task* task, const b2_env_config* config, b2_env** out);
/* Resets the rows with mask[i] != 0 (all rows if mask is NULL) to the initial state: steps 0, at_goal, counts and
 * count (if set). Draw counters are kept. */
b2_status b2_env_reset(b2_env* env, const b2_env_batch* batch, const uint8_t* mask, int32_t* count, void* stream);
/* One step of every row: actions[rows] (int64, device; NULL: the random policy). */
b2_status b2_env_step(b2_env* env, const b2_env_batch* batch, const b2_step_out* out, const int64_t* actions,
                      void* stream);
/* b2_env_step with next_task_ids[rows] (int32, device; NULL: none), the task an autoresetting row restarts in
 * (cuda::DeviceEnv::step, include/mymyr/cuda/env.hpp:180-184). The env has one task, id 0: another id, in any row, is
 * reported by b2_env_check_errors (B2_INVALID_ARGUMENT) and the rows keep their task. */
b2_status b2_env_step_ex(b2_env* env, const b2_env_batch* batch, const b2_step_out* out, const int64_t* actions,
                         const int32_t* next_task_ids, void* stream);
/* The env's device status since the last check (synchronizes the device; the status is cleared once reported):
 * B2_DEVICE_FAULT when a step found a state whose count cache did not match it (states written without a reset),
 * B2_INVALID_ARGUMENT for next_task_ids outside the env's tasks. */
b2_status b2_env_check_errors(b2_env* env);
void b2_env_destroy(b2_env* env);

#ifdef __cplusplus
}
#endif
#endif /* MYMYR_B200_H */
