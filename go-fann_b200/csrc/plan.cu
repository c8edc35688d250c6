// plan.cu — host-side routing of AND-of-labels queries into route tables
// (no device work).
//
// The reference plans each batch on the host before its search window
// (validate_and_prepare_queries, src/data/dataloader.cpp:10972, routing mode
// greedy_min_posting :7833-7836, predicate compile route_predicate::compile,
// src/planning/route_predicate_plan.h:175-315): a query's route is its label
// with the smallest posting list; a label that has a graph group becomes a
// graph route seeded at the group's seed row, any other label a posting
// route over its posting list; the rest of the conjunction -- the labels
// other than the route's own, which every row of the route carries -- is
// compiled into one DNF clause, enabled when it is not empty.  This is that
// loop in C++ for whole batches, writing the gofann_routes tables directly.
#include <cstring>

#include "common.cuh"

extern "C" {

int gofann_plan_categorical(const uint64_t* q_indptr, const uint32_t* q_labels, uint32_t n_queries,
                            const uint32_t* label_card, const int64_t* label_group, const uint32_t* group_seed,
                            const uint64_t* label_posting_begin, uint32_t n_labels, uint32_t n_groups,
                            gofann_plan_tables* graph, gofann_plan_tables* post)
{
    using gofann::fail;
    if (!q_indptr || (!q_labels && n_queries && q_indptr[n_queries]) || !label_card || !label_group || !group_seed ||
        !label_posting_begin || !graph || !post)
        return fail(GOFANN_ERR_INVALID, "plan_categorical: null argument");
    gofann_plan_tables* t[2] = {graph, post};
    for (gofann_plan_tables* x : t) {
        if (!x->query || !x->group_id || !x->start_local || !x->primary_label || !x->qlabel_indptr ||
            !x->qlabel_indices || !x->pred_handles || !x->clauses || !x->pred_enabled || !x->posting_begin ||
            !x->posting_count)
            return fail(GOFANN_ERR_INVALID, "plan_categorical: output table arrays missing");
        x->n_routes = x->n_labels = x->n_handles = 0;
        x->qlabel_indptr[0] = 0;
    }
    const uint64_t nnz = n_queries ? q_indptr[n_queries] : 0;
    for (uint32_t q = 0; q < n_queries; ++q) {
        const uint64_t b = q_indptr[q], e = q_indptr[q + 1];
        if (e < b || e > nnz) return fail(GOFANN_ERR_INVALID, "plan_categorical: query %u label range invalid", q);
        if (e == b) return fail(GOFANN_ERR_INVALID, "plan_categorical: query %u has no label", q);
        // the label with the smallest posting (the first one on ties)
        uint32_t lab = q_labels[b];
        if (lab >= n_labels) return fail(GOFANN_ERR_INVALID, "plan_categorical: label %u out of range", lab);
        for (uint64_t i = b + 1; i < e; ++i) {
            const uint32_t l = q_labels[i];
            if (l >= n_labels) return fail(GOFANN_ERR_INVALID, "plan_categorical: label %u out of range", l);
            if (label_card[l] < label_card[lab]) lab = l;
        }
        const int64_t grp = label_group[lab];
        if (grp >= static_cast<int64_t>(n_groups))
            return fail(GOFANN_ERR_INVALID, "plan_categorical: group %lld out of range", static_cast<long long>(grp));
        gofann_plan_tables& x = grp >= 0 ? *graph : *post;
        const uint32_t r = x.n_routes++;
        x.query[r] = q;
        x.group_id[r] = grp >= 0 ? static_cast<uint32_t>(grp) : 0u;
        x.start_local[r] = grp >= 0 ? group_seed[grp] : 0u;
        x.primary_label[r] = lab;
        x.posting_begin[r] = grp >= 0 ? 0u : label_posting_begin[lab];
        x.posting_count[r] = grp >= 0 ? 0u : label_card[lab];
        gofann_clause c{};
        c.label_begin = x.n_handles;
        for (uint64_t i = b; i < e; ++i) {
            x.qlabel_indices[x.n_labels++] = q_labels[i];
            if (q_labels[i] != lab) x.pred_handles[x.n_handles++] = q_labels[i];
        }
        c.label_end = x.n_handles;
        x.clauses[r] = c;
        x.pred_enabled[r] = c.label_end > c.label_begin ? 1 : 0;
        x.qlabel_indptr[r + 1] = x.n_labels;
    }
    return GOFANN_OK;
}

}  // extern "C"
