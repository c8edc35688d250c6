/* gofann_oracle.h — TEST INFRASTRUCTURE ONLY: CPU parity oracle of the
 * filtered-ANN search path.  Loaded by tests/, __graft_entry__.smoke() and
 * bench.py's CPU legs; never by the product library. */
#ifndef GOFANN_ORACLE_H
#define GOFANN_ORACLE_H
#include "../include/gofann.h"

#ifdef __cplusplus
extern "C" {
#endif

float oracle_warp_sum(const float* lanes);
void oracle_pq_build_lut(const float* queries, uint32_t n, uint32_t dim, const float* centroids,
                         uint32_t pq_dim, float* lut);
float oracle_pq_adc_one(const float* lut_row, uint32_t pq_dim, const uint8_t* code);
void oracle_pq_adc(const float* lut, uint32_t pq_dim, const uint8_t* codes, const uint32_t* pair_row,
                   const uint32_t* pair_sample, uint32_t n_pairs, float* out);
void oracle_pq_encode(const float* vectors, uint32_t n, uint32_t dim, const float* centroids,
                      uint32_t pq_dim, uint8_t* codes);
void oracle_rabitq_quantize(const float* rotated, uint32_t n, uint32_t padded_dim, int8_t* q8,
                            float* scale_out, float* k1_out);
int32_t oracle_rabitq_ip(const uint8_t* code, const int8_t* q8, uint32_t padded_dim);
float oracle_rabitq_combine(int32_t ip, float scale, float k1, float f_add, float f_rescale,
                            float gdist);
void oracle_rabitq_score(const gofann_codes* c, const gofann_prepared* p, const uint32_t* pair_row,
                         const uint32_t* pair_sample, uint32_t n_pairs, float* out, int32_t* ip_out);
void oracle_rabitq_encode(const float* residual, const float* rotated_centroid, uint32_t n,
                          uint32_t padded_dim, const uint32_t* anchor_ids, uint8_t* codes,
                          float* factors);
int oracle_hash_test(const uint32_t* t, uint32_t v);
int oracle_pickup_index(const float* keys, const uint32_t* vals, int size);
void oracle_rabitq_encode_f32(const float* residual, const float* rotated_centroid, uint32_t n,
                              uint32_t padded_dim, const uint32_t* anchor_ids, uint32_t* codes, float* factors);
int oracle_hash_add(uint32_t* t, uint32_t v);
int oracle_pred_enabled(const gofann_routes* r, uint32_t route);
int oracle_pred_matches(const gofann_routes* r, const gofann_attrs* a, uint32_t route, uint32_t sample);
int oracle_labels_match(const gofann_routes* r, const gofann_attrs* a, uint32_t route, uint32_t sample);
int oracle_beam_search(const gofann_graph* g, const gofann_attrs* a, const gofann_codes* c,
                       const gofann_prepared* p, const gofann_routes* r,
                       const gofann_search_params* sp, uint32_t* ids, float* d, int32_t* steps,
                       uint32_t* counters, int threads);
int oracle_beam_search_traced(const gofann_graph* g, const gofann_attrs* a, const gofann_codes* c,
                              const gofann_prepared* p, const gofann_routes* r,
                              const gofann_search_params* sp, uint32_t* ids, float* d, int32_t* steps,
                              uint32_t* counters, int threads, uint32_t* trace, uint32_t trace_width);
int oracle_posting_scan(const gofann_codes* c, const gofann_prepared* p, const gofann_attrs* a,
                        const gofann_routes* r, int scorer, const uint32_t* posting_ids,
                        const uint64_t* route_begin, const uint32_t* route_count, int k,
                        int score_first, uint32_t* out_ids, float* out_d);
float oracle_exact_l2(const void* base, int dtype, uint32_t dim, uint32_t sample, const void* query,
                      uint32_t row);
int oracle_rerank(const void* base, int dtype, uint32_t n_samples, uint32_t dim, const void* queries,
                  const gofann_attrs* a, const gofann_routes* r, const uint32_t* cand,
                  uint32_t width, int k, uint32_t* out_ids, float* out_d);
int oracle_route_merge(const uint32_t* ids, const float* d, uint32_t width, const uint32_t* qoff,
                       const uint32_t* qroutes, uint32_t nq, int k, uint32_t* out_ids, float* out_d);
int oracle_shard_merge(const uint32_t* ids, const float* d, uint32_t shards, uint32_t nq, int k,
                       uint32_t* out_ids, float* out_d);
int oracle_filtered_topk(const void* base, int dtype, uint32_t n_samples, uint32_t dim,
                         const void* queries, const gofann_attrs* a, const gofann_routes* r, int k,
                         uint32_t* out_ids, double* out_d);
int oracle_sl_can_enter(float dist, uint32_t id, const float* d, const uint32_t* ids, int k);
void oracle_sl_insert(float dist, uint32_t id, float* d, uint32_t* ids, int k);
void oracle_sl_sort(float* d, uint32_t* ids, int k);
int oracle_seq_smmh(const int* op, const float* key, const uint32_t* payload, int n,
                    float* out_first, uint32_t* out_second, uint32_t* popped);
int oracle_seq_result_heap(const float* key, const uint32_t* payload, int n, int cap,
                           float* out_first, uint32_t* out_second);
float oracle_full_l2(const void* base, int dtype, uint32_t dim, uint32_t sample, const void* queries,
                     uint32_t row);
int oracle_exact_search(const gofann_graph* g, const uint32_t* label_size, const gofann_attrs* a,
                        const void* base, int dtype, uint32_t dim, const void* queries, const gofann_routes* r,
                        const gofann_search_params* sp, uint32_t* ids, float* d, int32_t* steps,
                        uint32_t* trace, uint32_t trace_width, int threads);
int oracle_exact_posting_scan(const void* base, int dtype, uint32_t dim, const void* queries,
                              const gofann_attrs* a, const gofann_routes* r, const uint32_t* posting_ids,
                              const uint64_t* route_begin, const uint32_t* route_count, int k,
                              uint32_t* out_ids, float* out_d);
uint32_t oracle_levenshtein(const uint8_t* p, uint32_t m, const uint8_t* t, uint32_t n);
int oracle_full_pickup_index(const float* keys, const uint32_t* vals, int size);
void oracle_seq_hash(const uint32_t* values, int n, uint32_t* table, int32_t* outcome);

#ifdef __cplusplus
}
#endif
#endif
