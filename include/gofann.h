/*
 * gofann.h — C ABI of the B200 filtered-ANN search path.
 *
 * Every entry point takes plain pointers, sizes and a CUDA stream passed as
 * `void*` (NULL = legacy default stream).  Pointers documented as "device"
 * must be device-resident (cudaMalloc / torch CUDA storage); pointers
 * documented as "host" are ordinary host memory.  No entry point throws; each
 * returns a gofann_status (0 = success, negative = error) and records a
 * message readable through gofann_last_error() on the calling thread.
 *
 * The interfaces replace, one for one, the device halves of the reference's
 * search backends (putatio13/GO-FANN):
 *   gofann_pq_build_lut       computePQTable          src/search/pq/backend_pq.cu:1999-2022
 *   gofann_pq_adc             PQ neighbour scoring    src/search/pq/backend_pq.cu:4711-4725
 *   gofann_pq_encode          pq::transform (encode)  tools/quantization/pq_builder.cu:125-151
 *   gofann_rabitq_quantize    quantize_rabitq_queries_int8_kernel + compute_rabitq_query_factors_kernel
 *                                                     src/search/rabitq/backend_rabitq.cu:2898-2964
 *   gofann_rabitq_rotate      RabitqQueryRotation::apply  src/search/rabitq/rabitq_query_rotation.cuh:71-87
 *   gofann_rabitq_centroid_dist_tc  RabitqQueryRotation::centroid_distances  rabitq_query_rotation.cuh:89-113
 *   gofann_rabitq_encode      RaBitQ quantizer (cuVS fork) third_party/cuvs_rabitq/src/neighbors/ivf_rabitq/
 *                                                     gpu_index/quantizer_gpu_fast.cu:180-270
 *   gofann_rabitq_score       score_rabitq_code_device<kUseInt8Score=true>
 *                                                     src/search/rabitq/backend_rabitq.cu:3100-3200
 *   gofann_beam_search        native_warp_independent_search_kernel_impl (device-resident)
 *                                                     src/search/pq/backend_pq.cu:3988-5199,
 *                             native_rabitq_search_kernel src/search/rabitq/backend_rabitq.cu:3496-4299
 *   gofann_segment_merge      posting_segments::merge_shortlists
 *                                                     src/search/common/posting_segment_merge.cuh:13-61
 *   gofann_search_batch       execute_graph_batch + lowfreq scan + rerank + merge
 *                                                     src/search/pq/backend_pq.cu:9740-10185, 10769,
 *                                                     2479-2592, 13205-13226
 *   gofann_predicate_pass_masks  prepare_candidate_pass_masks
 *                                                     src/predicates/gpu_predicate_parallel.cuh:21-42
 *   gofann_posting_scan       lowfreq_pq_scan_kernel  src/search/pq/backend_pq.cu:2046-2185,
 *                             lowfreq_rabitq_scan_kernel src/search/rabitq/backend_rabitq.cu:5396-5751
 *   gofann_rerank             resident_pq_batch_exact_rerank_kernel src/search/pq/backend_pq.cu:5201-5310,
 *                             highfreq_float_gpu_l2/topk_kernel src/search/rabitq/backend_rabitq.cu:6173-6270,
 *                             highfreq_host_batch_rerank_range src/search/pq/backend_pq.cu:2479-2592
 *   gofann_route_merge        merge_route_results_to_original src/search/rabitq/rabitq_lowfreq_merge.h:710-815
 *   gofann_shard_merge        (no reference counterpart: the reference is single-GPU; the merge
 *                             order is the (dist, id) rule of rabitq_lowfreq_merge.h:800-806)
 *   gofann_exact_search       run_full_gpu_highfreq_route src/search/full_gpu/backend_full_gpu.cu:1682-2043
 *   gofann_exact_posting_scan full_gpu_lowfreq_kernel src/search/full_gpu/backend_full_gpu.cu:2124-2260
 *   gofann_plan_categorical   greedy_min_posting routing + route_predicate::compile (host)
 *                                                     src/data/dataloader.cpp:7833, 10972;
 *                                                     src/planning/route_predicate_plan.h:175-315
 */
#ifndef GOFANN_H
#define GOFANN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GOFANN_ABI_VERSION 4

#if defined(__GNUC__)
#define GOFANN_API __attribute__((visibility("default")))
#else
#define GOFANN_API
#endif

typedef enum gofann_status {
    GOFANN_OK = 0,
    GOFANN_ERR_INVALID = -1,     /* bad argument / shape / null pointer */
    GOFANN_ERR_CUDA = -2,        /* a CUDA runtime call failed */
    GOFANN_ERR_UNSUPPORTED = -3, /* shape outside the compiled limits */
    GOFANN_ERR_CAPACITY = -4,    /* a device capacity was exceeded */
    GOFANN_ERR_TIMEOUT = -5      /* a bounded device wait ran out */
} gofann_status;

/* Compiled limits (backend_pq.cu:66-75, runtime_defaults.h:30-52). */
#define GOFANN_MAX_DEGREE 64
#define GOFANN_MAX_QUEUE 512
#define GOFANN_MAX_TOPK 10
#define GOFANN_MAX_RESULT_WIDTH 512
#define GOFANN_MAX_SHORTLIST 400
#define GOFANN_PQ_CENTROIDS 256
#define GOFANN_HASH_CAPACITY 4096

enum { GOFANN_EARLY_STOP_FIXED = 0, GOFANN_EARLY_STOP_OFF = 1, GOFANN_EARLY_STOP_ADAPTIVE = 2 };
enum { GOFANN_SCORER_PQ = 0, GOFANN_SCORER_RABITQ = 1 };
enum { GOFANN_DTYPE_U8 = 0, GOFANN_DTYPE_F32 = 1, GOFANN_DTYPE_F16 = 2 };
/* PQ scoring inside the traversal: read a prebuilt LUT from global memory,
 * stage it in shared memory per route, or evaluate each table entry from the
 * query and the codebook where it is used (no per-query table at all).
 * GOFANN_PQ_U8: u8 queries and a codebook whose values are integers in
 * 0..255 (checked on the device: any other value sets the status word to
 * GOFANN_ERR_INVALID and nothing is searched).  Every table entry and every
 * partial sum of the reference's float ADC is then an integer below 2^24,
 * exact in float whatever the order, so the distance is scored as an integer
 * sum of byte differences (absolute difference + dot product of packed
 * bytes) against a packed copy of the codebook in shared memory: the same
 * bits as the table modes, no per-query table. */
enum { GOFANN_PQ_LUT_GLOBAL = 0, GOFANN_PQ_LUT_SHARED = 1, GOFANN_PQ_DIRECT = 2, GOFANN_PQ_U8 = 3 };

/* DNF clause over label handles and range atoms (gpu_predicate_index.cuh:24-25). */
typedef struct gofann_clause {
    uint32_t label_begin, label_end, range_begin, range_end;
} gofann_clause;

/* Range atom: mode 0 any, 1 v>lower, 2 v<upper, 3 lower<=v<upper (range_filter.cuh:28-45). */
typedef struct gofann_range_atom {
    uint32_t dimension, mode;
    float lower, upper;
} gofann_range_atom;

/* String atom of a DNF clause: the sample's string attribute equals the
 * query string (GOFANN_STRING_EXACT), or is within max_edits insertions,
 * deletions and substitutions of it (GOFANN_STRING_FUZZY, Levenshtein
 * distance).  The query string is pred_string_bytes[offset, offset +
 * length).  A fuzzy atom's query string has at most 32 bytes, all below 128,
 * and its row of pred_string_peq holds gofann_string_peq() of it.  The
 * reference has no edit-distance predicate (it rewrites fuzzy queries into
 * token labels, src/data/dataloader.cpp:2973-3010); this is the device check
 * its configurations call for. */
enum { GOFANN_STRING_EXACT = 0, GOFANN_STRING_FUZZY = 1 };
#define GOFANN_FUZZY_MAX_LENGTH 32
typedef struct gofann_string_atom {
    uint32_t kind, max_edits, offset, length;
} gofann_string_atom;

/* Integer range atom over an int64 attribute column: mode 0 any, 1
 * v>lower, 2 v<upper, 3 lower<=v<upper (the float atom's modes, exact on
 * int64 values; the reference compares float32, range_filter.cuh:28-45). */
typedef struct gofann_int_atom {
    uint32_t dimension, mode;
    int64_t lower, upper;
} gofann_int_atom;

/* Further atoms of clause i (parallel to the clauses array): string atoms
 * [string_begin, string_end) of pred_strings and integer atoms [int_begin,
 * int_end) of pred_ints, ANDed with the clause's labels and float ranges. */
typedef struct gofann_clause_ext {
    uint32_t string_begin, string_end, int_begin, int_end;
} gofann_clause_ext;

/* Concatenated per-label graphs: row = label_offset[group] + local_row
 * (GraphRuntime::graph + GraphMetadata, dataloader.h:583-602,753-836). */
typedef struct gofann_graph {
    const uint32_t* adjacency;       /* device [total_rows][degree], UINT32_MAX padding */
    const uint32_t* row_to_sample;   /* device [total_rows] */
    const uint64_t* row_filter_mask; /* device [total_rows], or NULL = implicit all-ones */
    const uint32_t* label_offset;    /* device [group_count] */
    uint32_t total_rows;
    uint32_t degree;
    uint32_t group_count;
    uint32_t reserved;
    /* Optional per-row records (gofann_build_row_records), or NULL: row r at
     * records + r * record_stride holds the PQ code row of its sample
     * (pq_dim bytes), then at byte GOFANN_RECORD_META(pq_dim) four uint32:
     * the sample id, the start and the length of its label-CSR row, and the
     * row's label signature (GOFANN_LABEL_SIG_BIT of every label OR-ed
     * together), then, 16 bytes further, the label row itself when it has at
     * most GOFANN_RECORD_INLINE_LABELS labels.  One 128-byte line per row at
     * config-2 shape: scoring and predicate checks of a candidate read one
     * line instead of following row -> sample -> code and sample -> CSR
     * offsets -> labels, and a candidate whose signature lacks a bit of the
     * route's clause skips the label row.  Results are the same with or
     * without records; records must come from gofann_build_row_records of
     * this ABI version. */
    const uint8_t* records;
    uint32_t record_stride;          /* bytes, a multiple of 16 */
    uint32_t reserved2;
} gofann_graph;

/* Byte offset of a record's (sample, label start, label length, label
 * signature) words. */
#define GOFANN_RECORD_META(pq_dim) ((((pq_dim) + 15u) / 16u) * 16u)
/* Label rows of at most this many labels are stored in the record. */
#define GOFANN_RECORD_INLINE_LABELS 16u
/* Signature bit of a label: one of 32, from a multiplicative hash.  A row
 * can carry every label of a clause only if its signature holds all their
 * bits. */
#define GOFANN_LABEL_SIG_BIT(label) (1u << ((((uint32_t)(label)) * 0x9E3779B1u) >> 27))

/* Per-sample attributes: sample-major label CSR (sorted, unique per row) and
 * float range values (SparseLabelMatrix / base_range_values). */
typedef struct gofann_attrs {
    const uint64_t* label_indptr;  /* device [n_samples+1] */
    const uint32_t* label_indices; /* device [nnz] */
    const float* range_values;     /* device [n_samples][range_count] or NULL */
    uint32_t n_samples;
    uint32_t range_count;
    /* one string per sample: bytes string_bytes[string_offsets[s],
     * string_offsets[s+1]) (device, or NULL when no clause has string atoms) */
    const uint64_t* string_offsets;
    const uint8_t* string_bytes;
    const int64_t* int_values;     /* device [n_samples][int_count] or NULL */
    uint32_t int_count;
    uint32_t reserved;
} gofann_attrs;

/* Navigation codes.  PQ: uint8 [n][pq_dim] (pq.codes.bin rows).  RaBitQ:
 * 1-bit codes [n][padded_dim/8] stored as little-endian uint32 words with
 * dimension d at bit 31-(d%32) of word d/32, factors [n][3] = (f_add,
 * f_rescale, f_err), anchor ids [n] (RabitqArtifactHeader v2 payload). */
typedef struct gofann_codes {
    const uint8_t* pq_codes;
    uint32_t pq_dim;
    uint32_t n_samples;
    const uint8_t* rq_codes;
    const float* rq_factors;
    const uint32_t* rq_anchor_ids;
    uint32_t padded_dim;
    uint32_t num_anchors;
} gofann_codes;

/* Per-query prepared state.  PQ: either the lookup tables lut
 * [n_rows][pq_dim][256], or the raw query rows pq_query [n_rows][dim] (u8 or
 * f32, pq_query_dtype) with the codebook pq_centroids [256][dim] -- then every
 * table entry is evaluated where it is used, with the same fma order, which
 * gives the same bits.  RaBitQ: int8 query [n_rows][padded_dim], scale
 * [n_rows], k1xsumq [n_rows], centroid distances [n_rows][num_anchors]. */
typedef struct gofann_prepared {
    const float* pq_lut;
    const int8_t* rq_q8;
    const float* rq_scale;
    const float* rq_k1xsumq;
    const float* rq_centroid_dist;
    uint32_t n_rows;
    uint32_t reserved;
    const void* pq_query;
    const float* pq_centroids;
    int32_t pq_query_dtype; /* GOFANN_DTYPE_U8 or GOFANN_DTYPE_F32 */
    uint32_t dim;
} gofann_prepared;

/* Routed queries (GraphRuntime route tables + gpu_predicate::View).  Every
 * per-route pointer except query_row, group_id and start_local may be NULL. */
typedef struct gofann_routes {
    uint32_t n_routes;
    uint32_t range_count;
    const uint32_t* query_row;   /* route -> row of gofann_prepared */
    const uint32_t* group_id;    /* route -> graph group (query_group_ids) */
    const uint32_t* start_local; /* route -> seed local row (start_local_ids) */
    const uint64_t* filter_bits; /* route -> query_filter_bits; NULL = always match */
    const uint8_t* range_modes;  /* [n_routes][range_count] */
    const float* range_lower;
    const float* range_upper;
    /* residual label check (resident_pq_labels_match, backend_pq.cu:3934-3965) */
    const uint64_t* qlabel_indptr;  /* [n_routes+1] */
    const uint32_t* qlabel_indices; /* labels every result must carry */
    const uint32_t* primary_label;  /* [n_routes] label covered by the route itself */
    /* compiled DNF predicate (gpu_predicate::View with clauses) */
    const uint32_t* pred_offsets;   /* [n_routes+1] into clauses, or NULL = no predicate */
    const gofann_clause* clauses;
    const uint32_t* pred_handles;
    const gofann_range_atom* pred_ranges;
    const uint8_t* pred_enabled;    /* [n_routes] or NULL = enabled iff pred_offsets */
    const uint8_t* route_compiled;  /* [n_routes] or NULL */
    /* string and integer atoms of the clauses (NULL pred_ext = none) */
    const gofann_clause_ext* pred_ext;
    const gofann_string_atom* pred_strings;
    const uint8_t* pred_string_bytes;
    const uint32_t* pred_string_peq; /* [n_string_atoms][128], rows of fuzzy atoms filled */
    const gofann_int_atom* pred_ints;
} gofann_routes;

typedef struct gofann_search_params {
    int32_t queue_size;      /* beam / search_queue_size, 1..512 */
    int32_t stop_width;      /* topk used by the stop rule, 1..10 */
    int32_t result_width;    /* shortlist emitted per route, 1..512 */
    int32_t finish_limit;    /* search_finish_count (fixed mode) */
    int32_t early_stop_mode; /* GOFANN_EARLY_STOP_* */
    int32_t max_steps;       /* 0 = unlimited */
    int32_t scorer;          /* GOFANN_SCORER_* */
    int32_t predicate_bias;  /* 1 = penalise frontier entries failing the DNF */
    float alpha;             /* predicate_bias_alpha */
    int32_t pending_base_stop;
    int32_t full_label_check;     /* 1 = resident residual label check on expansion */
    int32_t pq_mode;              /* PQ scoring: GOFANN_PQ_LUT_GLOBAL, _LUT_SHARED, _DIRECT or _U8 */
    int32_t resident_warps;       /* cap on concurrently running routes (warps) of the persistent
                                     grid; 0 = automatic: as many as fit on the SMs, reduced in
                                     GOFANN_PQ_LUT_GLOBAL mode so that the per-route tables in
                                     flight stay L2-resident */
} gofann_search_params;

/* Per-route device counters written by gofann_beam_search (may be NULL):
 * [n_routes][4] = expanded nodes, distance evaluations, predicate probes,
 * frontier admissions. */
typedef struct gofann_search_out {
    uint32_t* ids;      /* device [n_routes][result_width], UINT32_MAX fill */
    float* dists;       /* device [n_routes][result_width], FLT_MAX fill */
    int32_t* steps;     /* device [n_routes] or NULL */
    uint32_t* counters; /* device [n_routes][4] or NULL */
    int32_t* status;    /* device [1] error word or NULL */
    /* optional expansion trace (expansion_trace::View, src/profiling/
     * expansion_trace.h:19): the first trace_width expanded local rows of
     * each route in expansion order, UINT32_MAX fill; NULL = off */
    uint32_t* trace;
    uint32_t trace_width;
    uint32_t reserved;
} gofann_search_out;

/* ---------------------------------------------------------------- basics */
GOFANN_API int gofann_abi_version(void);
/* Host helper (no device work): the 128-entry match table of a fuzzy string
 * atom -- bit i of peq_out[c] is set when pattern[i] == c -- for the
 * bit-parallel edit distance of Myers (J. ACM 46(3), 1999) that the device
 * check runs.  length <= GOFANN_FUZZY_MAX_LENGTH, bytes below 128. */
GOFANN_API int gofann_string_peq(const uint8_t* pattern, uint32_t length, uint32_t* peq_out);
GOFANN_API const char* gofann_last_error(void);
/* Number of streaming multiprocessors of the current device (0 on error). */
GOFANN_API int gofann_device_sm_count(void);

/* ------------------------------------------------------------- PQ stages */
/* LUT [n][pq_dim][256]: sum over the subvector of fma(diff, diff, acc) with
 * diff = q - c, sequential in d (computePQTable, backend_pq.cu:1999-2022).
 * queries: device [n][dim] of dtype u8 or f32; centroids: device [256][dim]
 * (pivots + mean, backend_pq.cu:1812-1815). */
GOFANN_API int gofann_pq_build_lut(const void* queries, int query_dtype, uint32_t n, uint32_t dim,
                        const float* centroids, uint32_t pq_dim, float* lut_out, void* stream);

/* ADC for n_pairs (query row, sample) pairs with the reference's warp order:
 * lane j sums subspaces j, j+32 sequentially, then an xor butterfly
 * 16,8,4,2,1 (backend_pq.cu:4711-4725). */
GOFANN_API int gofann_pq_adc(const float* lut, uint32_t pq_dim, const uint8_t* codes,
                  const uint32_t* pair_row, const uint32_t* pair_sample, uint32_t n_pairs,
                  float* dist_out, void* stream);

/* Nearest-centroid PQ encoding (argmin, lowest centroid index on ties). */
GOFANN_API int gofann_pq_encode(const void* vectors, int dtype, uint32_t n, uint32_t dim,
                     const float* centroids, uint32_t pq_dim, uint8_t* codes_out, void* stream);

/* --------------------------------------------------------- RaBitQ stages */
/* From rotated queries [n][padded_dim] (f32): int8 query, scale =
 * max|q|/127 (1 if 0), q8 = clamp(rint(q/scale), -127, 127), k1xsumq =
 * -0.5*sum(q) (backend_rabitq.cu:2898-2964). */
GOFANN_API int gofann_rabitq_quantize(const float* rotated, uint32_t n, uint32_t padded_dim,
                           int8_t* q8_out, float* scale_out, float* k1xsumq_out, void* stream);

/* gdist[q][a] = max(0, |q|^2 + |c_a|^2 - 2 q.c_a) (rabitq_query_rotation.cuh:89-113). */
GOFANN_API int gofann_rabitq_centroid_dist(const float* rotated, uint32_t n, const float* anchors,
                                uint32_t num_anchors, uint32_t padded_dim, float* gdist_out,
                                void* stream);

/* Precision of the tensor-core preparation GEMMs: GOFANN_GEMM_TF32 = one
 * TF32 pass (index-time use), GOFANN_GEMM_TF32X3 = three TF32 passes on the
 * split operands (x = tf32(x) + tf32(x - tf32(x))), FP32-accurate to the
 * reference's tolerance (rabitq_query_rotation_test.cu:30-32, 48-50). */
enum { GOFANN_GEMM_TF32 = 0, GOFANN_GEMM_TF32X3 = 1 };

/* Bytes of device scratch (256-byte aligned) for one preparation GEMM of
 * `rows` x `k` by `cols` x `k`: the prepared operands and two norm vectors. */
GOFANN_API size_t gofann_rabitq_gemm_scratch_bytes(uint32_t rows, uint32_t k, uint32_t cols, int precision);

/* Query rotation q' = q . R (RabitqQueryRotation::apply,
 * rabitq_query_rotation.cuh:71-87) on the tensor cores (tcgen05, TMA):
 * queries device [n][dim] f32, rotation device [dim][padded_dim] f32 (row
 * major, as the reference stores it; padded_dim >= dim), rotated_out device
 * [n][padded_dim].  scratch (256-byte aligned): gofann_rabitq_gemm_scratch_bytes(n, dim,
 * padded_dim, precision).  status (device, may be NULL) is set to
 * GOFANN_ERR_TIMEOUT if a bounded device wait ran out. */
GOFANN_API int gofann_rabitq_rotate(const float* queries, uint32_t n, uint32_t dim, const float* rotation,
                                    uint32_t padded_dim, int precision, float* rotated_out, void* scratch,
                                    size_t scratch_bytes, int32_t* status, void* stream);

/* Centroid distances on the tensor cores (RabitqQueryRotation::
 * centroid_distances, rabitq_query_rotation.cuh:89-113): gdist[q][a] =
 * max(0, -2 q'.c_a + |q'|^2 + |c_a|^2) for rotated queries [n][padded_dim]
 * and anchors [num_anchors][padded_dim].  scratch:
 * gofann_rabitq_gemm_scratch_bytes(n, padded_dim, num_anchors, precision). */
GOFANN_API int gofann_rabitq_centroid_dist_tc(const float* rotated, uint32_t n, const float* anchors,
                                              uint32_t num_anchors, uint32_t padded_dim, int precision,
                                              float* gdist_out, void* scratch, size_t scratch_bytes,
                                              int32_t* status, void* stream);

/* 1-bit RaBitQ encoder (index time; quantizer_gpu_fast.cu:180-270 of the
 * reference's cuVS RaBitQ fork): residuals [n][padded_dim] = (x - c) R,
 * rotated centroids [num_anchors][padded_dim] and each vector's anchor ->
 * codes [n][padded_dim/8] (4-byte aligned; layout of gofann_codes) and
 * factors [n][3] = (f_add, f_rescale, f_err).  FP32 in a fixed order (lane
 * partials over dimensions l, l+32, ..., xor butterfly, formulas left to
 * right), bit-exact to the CPU oracle given the residuals. */
GOFANN_API int gofann_rabitq_encode(const float* residual, const float* rotated_centroids,
                                    const uint32_t* anchor_ids, uint32_t n, uint32_t padded_dim,
                                    uint8_t* codes_out, float* factors_out, void* stream);

/* Entry rows of graph routes (no counterpart in the reference, whose routes
 * start at a fixed row per graph): start_local_out[r] =
 * anchor_entry[argmin_a gdist[query_row[r]][a]] (lowest anchor on ties),
 * i.e. each route starts at the entry row of its query's nearest anchor.
 * gdist device [rows][num_anchors] (gofann_rabitq_centroid_dist_tc),
 * anchor_entry device [num_anchors] (a row of each anchor's cluster). */
GOFANN_API int gofann_rabitq_route_entries(const float* gdist, uint32_t num_anchors, const uint32_t* query_row,
                                           uint32_t n_routes, const uint32_t* anchor_entry,
                                           uint32_t* start_local_out, void* stream);

/* 1-bit int8 estimator for pairs (backend_rabitq.cu:3100-3200):
 * est = (f_add + gdist) + f_rescale * (float(ip_int) * scale + k1xsumq). */
GOFANN_API int gofann_rabitq_score(const gofann_codes* codes, const gofann_prepared* prep,
                        const uint32_t* pair_row, const uint32_t* pair_sample, uint32_t n_pairs,
                        float* dist_out, int32_t* ip_int_out, void* stream);

/* ----------------------------------------------------------- traversal */
/* Bytes of device scratch gofann_beam_search needs for n_routes routes
 * (one 4096-slot visited table per resident warp). */
GOFANN_API size_t gofann_beam_search_scratch_bytes(uint32_t n_routes);

/* Filtered graph beam search, one warp per route (backend_pq.cu:3988-5013). */
GOFANN_API int gofann_beam_search(const gofann_graph* graph, const gofann_attrs* attrs,
                       const gofann_codes* codes, const gofann_prepared* prep,
                       const gofann_routes* routes, const gofann_search_params* params,
                       const gofann_search_out* out, void* scratch, size_t scratch_bytes,
                       void* stream);

/* Allocation-free variant of gofann_beam_search (no counterpart in the
 * reference, which allocates its traversal scratch with cudaMalloc).  For
 * callers that cannot allocate device memory themselves -- a host runtime or
 * database whose allocator owns the device, code that must not allocate
 * while a stream is being captured into a CUDA graph, latency-critical paths
 * -- the visited tables and route counter live in a static device array of
 * 16 MiB + 256 B inside the library (1,024 visited tables), held by every GPU
 * that loads the library until the process exits.  At most 1,024 warps run
 * at once; any number of routes is accepted.  The first call on each device
 * looks up the array's device address (make it before any stream capture
 * begins).  Calls share the array: calls whose kernels overlap on the GPU
 * race and must be serialised by the caller.  Results equal
 * gofann_beam_search's bit for bit. */
GOFANN_API int gofann_beam_search_noalloc(const gofann_graph* graph, const gofann_attrs* attrs,
                                          const gofann_codes* codes, const gofann_prepared* prep,
                                          const gofann_routes* routes, const gofann_search_params* params,
                                          const gofann_search_out* out, void* stream);

/* ------------------------------------------------ Full-GPU exact mode */
/* Bytes of device scratch gofann_exact_search needs for n_routes routes. */
GOFANN_API size_t gofann_exact_search_scratch_bytes(uint32_t n_routes);

/* Full-GPU exact-distance traversal (run_full_gpu_highfreq_route,
 * src/search/full_gpu/backend_full_gpu.cu:1682-2043): the graph routes are
 * searched with the exact L2 distance of the full base vectors (base device
 * [n_samples][dim] of dtype u8 / f32 / f16, queries device [n_rows][dim] of
 * the same dtype, both 16-byte aligned with rows a multiple of 16 bytes) --
 * no codes and no rerank.  Per route the result is the top-k (k =
 * params->result_width, 1..10) of the expanded nodes that pass the route's
 * filter (filter_bits against graph->row_filter_mask, the residual labels
 * qlabel_* except primary_label, and the range_modes atoms), as sample ids
 * ascending by (distance, id); the search stops by the reference's
 * finish-hit rule (params->early_stop_mode, finish_limit, max_steps).
 * label_size: device [group_count] rows per graph group, or NULL to derive
 * it from consecutive label_offset entries (the last group ends at
 * total_rows).  out->counters, when set, receive per route [expanded
 * nodes, distance evaluations, expanded nodes that passed the filter,
 * frontier admissions]. */
GOFANN_API int gofann_exact_search(const gofann_graph* graph, const uint32_t* label_size,
                                   const gofann_attrs* attrs, const void* base, int dtype, uint32_t dim,
                                   const void* queries, const gofann_routes* routes,
                                   const gofann_search_params* params, const gofann_search_out* out,
                                   void* scratch, size_t scratch_bytes, void* stream);

/* Full-GPU exact posting scan (full_gpu_lowfreq_kernel,
 * src/search/full_gpu/backend_full_gpu.cu:2124-2260): every member of each
 * route's posting slice that passes the route's DNF predicate is scored by
 * exact L2 (the same arithmetic as gofann_exact_search) and the k smallest
 * (distance, id) pairs are kept (UINT32_MAX / FLT_MAX fill).  out_*: device
 * [n_routes][k]. */
GOFANN_API int gofann_exact_posting_scan(const void* base, int dtype, uint32_t n_samples, uint32_t dim,
                                         const void* queries, const gofann_attrs* attrs,
                                         const gofann_routes* routes, const uint32_t* posting_ids,
                                         const uint64_t* route_begin, const uint32_t* route_count, int32_t k,
                                         uint32_t* out_ids, float* out_dists, void* stream);

/* ------------------------------------------------------- posting scans */
/* Brute-force scan of each route's posting slice [begin, begin+count) of
 * posting_ids, DNF filter (before scoring, or after a can-enter test when
 * score_first), top-shortlist_k by (dist, id) (backend_pq.cu:2046-2134). PQ
 * distances are sequential sums over subspaces (backend_pq.cu:2101-2104),
 * read from prep->pq_lut or from a table built per route from pq_query and
 * pq_centroids.  pq_mode GOFANN_PQ_U8 (u8 pq_query, 4-wide subvectors,
 * pq_dim a multiple of 16, dim <= 256) scores against the integer codebook
 * instead -- the same bits with no per-route table; a codebook value that
 * is not an integer in 0..255 sets *status (when non-NULL) to
 * GOFANN_ERR_INVALID and leaves every shortlist empty.  Any other pq_mode
 * uses the tables. */
GOFANN_API int gofann_posting_scan(const gofann_codes* codes, const gofann_prepared* prep,
                        const gofann_attrs* attrs, const gofann_routes* routes, int scorer,
                        const uint32_t* posting_ids, const uint64_t* route_begin,
                        const uint32_t* route_count, int32_t shortlist_k, int32_t score_first,
                        int32_t pq_mode, uint32_t* out_ids, float* out_dists, int32_t* status,
                        void* stream);

/* ------------------------------------------------------- whole batches */
/* Index-resident inputs of a batch (device pointers).  The PQ fields serve
 * GOFANN_SCORER_PQ, the rq_ fields GOFANN_SCORER_RABITQ (codes.rq_* hold
 * the 1-bit codes, factors and anchor ids). */
typedef struct gofann_index {
    gofann_graph graph;
    gofann_attrs attrs;
    gofann_codes codes;
    const float* pq_centroids;     /* [256][dim]: pivots + mean (backend_pq.cu:1812-1815) */
    const void* base;              /* rerank store [n_samples][dim] of base_dtype */
    int32_t base_dtype;            /* GOFANN_DTYPE_* */
    uint32_t dim;
    const uint32_t* posting_ids;   /* label postings and attribute-order slices */
    const float* rq_rotation;      /* [dim][padded_dim] */
    const float* rq_anchors;       /* [num_anchors][padded_dim], rotated */
    const uint32_t* rq_anchor_entry; /* [num_anchors] graph entry row of each anchor, or NULL */
} gofann_index;

/* One batch of routed queries (device pointers).  Route query_row values
 * index the query rows; results of route r land in slot r of [graph routes ;
 * posting routes], which query_route_offsets / query_routes group by query
 * (route_to_original_query). */
typedef struct gofann_batch {
    const void* queries;            /* [n_queries][dim]: u8 for a u8 base, f32 otherwise */
    uint32_t n_queries;
    uint32_t reserved;
    gofann_routes graph_routes;     /* traversal routes (n_routes may be 0) */
    gofann_routes posting_routes;   /* posting-scan routes (n_routes may be 0) */
    const uint64_t* posting_begin;  /* [posting n_routes] offsets into index posting_ids */
    const uint32_t* posting_count;
    const uint32_t* query_route_offsets; /* [n_queries+1] */
    const uint32_t* query_routes;
} gofann_batch;

typedef struct gofann_batch_params {
    gofann_search_params search;    /* traversal; search.result_width = traversal shortlist */
    int32_t posting_shortlist;      /* 1..400 */
    int32_t topk;                   /* results per query, 1..10 */
    int32_t rq_entries;             /* RaBitQ: 1 = start each graph route at the entry row of its
                                       query's nearest anchor (needs rq_anchor_entry) */
    int32_t reserved;
} gofann_batch_params;

/* Device scratch gofann_search_batch needs for this batch shape. */
GOFANN_API size_t gofann_search_batch_scratch_bytes(const gofann_index* index, const gofann_batch* batch,
                                                    const gofann_batch_params* params);

/* A whole batch on one stream with no allocation and no host
 * synchronisation: query preparation (PQ: the lookup tables in the table
 * modes; RaBitQ: rotation and centroid distances on the tensor cores,
 * int8 quantisation, optional route entry points), the traversal of the
 * graph routes, the posting scans, the exact rerank of both shortlist sets
 * and the route -> query merge -- execute_graph_batch,
 * run_lowfreq_pq_search_with_context, the high-frequency rerank and
 * merge_route_results_to_original (backend_pq.cu:9740-10185, 10769,
 * 2479-2592, 13205-13226; backend_rabitq.cu:13762-13776).  out_ids /
 * out_dists: device [n_queries][topk]; status: device [1] error word or
 * NULL.  Results equal the per-stage calls' bit for bit. */
GOFANN_API int gofann_search_batch(const gofann_index* index, const gofann_batch* batch,
                                   const gofann_batch_params* params, void* scratch, size_t scratch_bytes,
                                   uint32_t* out_ids, float* out_dists, int32_t* status, void* stream);

/* Merge of segment shortlists (merge_shortlists,
 * src/search/common/posting_segment_merge.cuh:13-61): a long posting or range
 * slice is scanned as several segments (one gofann_posting_scan route each,
 * shortlists [segments][shortlist_k]); route r owns segments seg_indptr[r] ..
 * seg_indptr[r+1] - 1 and gets the shortlist_k smallest (dist, id) pairs of
 * their union -- the shortlist one scan of the whole slice gives.  out_*:
 * device [n_routes][shortlist_k], UINT32_MAX / FLT_MAX fill. */
GOFANN_API int gofann_segment_merge(const uint32_t* seg_indptr, uint32_t n_routes, const uint32_t* seg_ids,
                                    const float* seg_dists, int32_t shortlist_k, uint32_t* out_ids,
                                    float* out_dists, void* stream);

/* ------------------------------------------------- predicate bitmaps */
/* Pass bits of candidate rows (prepare_candidate_pass_masks,
 * src/predicates/gpu_predicate_parallel.cuh:21-42): bit i % 32 of
 * out_masks[i / 32] is 1 when candidate i -- local row cand_rows[i] of the
 * graph group of route cand_route[i], i.e. the sample
 * row_to_sample[label_offset[group_id[route]] + row] -- matches the route's
 * DNF predicate (gpu_predicate::matches), or when the route has no enabled
 * predicate.  out_masks: device [ceil(n_candidates / 32)].  A route, group
 * or row out of range gives a 0 bit and sets *status (when non-NULL) to
 * GOFANN_ERR_INVALID. */
GOFANN_API int gofann_predicate_pass_masks(const gofann_graph* graph, const gofann_attrs* attrs,
                                           const gofann_routes* routes, const uint32_t* cand_route,
                                           const uint32_t* cand_rows, uint32_t n_candidates,
                                           uint32_t* out_masks, int32_t* status, void* stream);

/* ------------------------------------------------------ route planning */
/* Route tables written by gofann_plan_categorical (host arrays the caller
 * allocates: routes up to the batch's query count, labels and handles up to
 * its label count).  One DNF clause per route (pred_offsets = 0, 1, ..., the
 * caller's identity array); the counts are outputs. */
typedef struct gofann_plan_tables {
    uint32_t* query;           /* [routes] original query of the route (route_to_original_query) */
    uint32_t* group_id;        /* [routes] graph group, 0 for posting routes */
    uint32_t* start_local;     /* [routes] seed row of the group, 0 for posting routes */
    uint32_t* primary_label;   /* [routes] the label the route covers */
    uint64_t* qlabel_indptr;   /* [routes + 1] */
    uint32_t* qlabel_indices;  /* the query's labels, as given */
    uint32_t* pred_handles;    /* the residual labels (all but the primary one) */
    gofann_clause* clauses;    /* [routes] */
    uint8_t* pred_enabled;     /* [routes] 1 when the residual is not empty */
    uint64_t* posting_begin;   /* [routes] posting routes: the label's posting slice */
    uint32_t* posting_count;
    uint32_t n_routes, n_labels, n_handles, reserved;
} gofann_plan_tables;

/* Host-side routing of a batch of AND-of-labels queries (greedy_min_posting,
 * src/data/dataloader.cpp:7833-7836, in validate_and_prepare_queries
 * :10972; the residual compiled as in route_predicate::compile,
 * src/planning/route_predicate_plan.h:175-315): a query's route is its label
 * with the smallest label_card (the first on ties); a label with
 * label_group >= 0 gives a graph route seeded at group_seed[group], any other
 * a posting route over label_posting_begin / label_card.  Host pointers; no
 * device work. */
GOFANN_API int gofann_plan_categorical(const uint64_t* q_indptr, const uint32_t* q_labels, uint32_t n_queries,
                                       const uint32_t* label_card, const int64_t* label_group,
                                       const uint32_t* group_seed, const uint64_t* label_posting_begin,
                                       uint32_t n_labels, uint32_t n_groups, gofann_plan_tables* graph,
                                       gofann_plan_tables* post);

/* ---------------------------------------------------------- exact rerank */
/* Exact L2 of each candidate against its query row, residual label check
 * (every label of qlabel_indices except primary_label), duplicates dropped,
 * top-k ascending by (dist, id) (backend_pq.cu:2479-2592, 5201-5310).
 * base: device [n_samples][dim] of dtype; queries: device [n_rows][dim],
 * u8 for a u8 base, f32 otherwise. routes supplies query_row and the residual
 * label tables (may be NULL for no check). */
GOFANN_API int gofann_rerank(const void* base, int dtype, uint32_t n_samples, uint32_t dim,
                  const void* queries, const gofann_attrs* attrs, const gofann_routes* routes,
                  const uint32_t* cand_ids, uint32_t width, int32_t topk,
                  uint32_t* out_ids, float* out_dists, void* stream);

/* --------------------------------------------------------------- merges */
/* Route -> original query merge: dedup by id keeping the min distance, sort
 * by (dist, id), truncate to topk, UINT32_MAX / FLT_MAX fill
 * (rabitq_lowfreq_merge.h:710-815). query_route_offsets [n_queries+1] and
 * query_routes list the routes of each original query. */
GOFANN_API int gofann_route_merge(const uint32_t* route_ids, const float* route_dists, uint32_t width,
                       const uint32_t* query_route_offsets, const uint32_t* query_routes,
                       uint32_t n_queries, int32_t topk, uint32_t* out_ids, float* out_dists,
                       void* stream);

/* Shard merge: per query, n_shards sorted top-k lists (ids already global)
 * laid out [n_shards][n_queries][k] -> top-k by (dist, id). */
GOFANN_API int gofann_shard_merge(const uint32_t* shard_ids, const float* shard_dists, uint32_t n_shards,
                       uint32_t n_queries, int32_t topk, uint32_t* out_ids, float* out_dists,
                       void* stream);

/* Per-row records for the traversal (see gofann_graph.records): record_stride
 * = GOFANN_RECORD_META(pq_dim) + 16 + 4 * GOFANN_RECORD_INLINE_LABELS (128
 * bytes at pq_dim 48);
 * out: device [total_rows][record_stride].  Label CSR offsets must fit in
 * 32 bits (fails with GOFANN_ERR_UNSUPPORTED otherwise, checked on the
 * device through `status`, which may be NULL); a row whose row_to_sample
 * entry is not below attrs->n_samples gets an all-zero record and sets
 * `status` to GOFANN_ERR_INVALID. */
GOFANN_API size_t gofann_row_record_stride(uint32_t pq_dim);
GOFANN_API int gofann_build_row_records(const gofann_graph* graph, const gofann_attrs* attrs,
                                        const gofann_codes* codes, uint8_t* out, int32_t* status, void* stream);

/* Adds base to every id that is not UINT32_MAX (local -> global shard ids). */
GOFANN_API int gofann_offset_ids(uint32_t* ids, size_t n, uint32_t base, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GOFANN_H */
