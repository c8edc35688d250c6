// batch_driver.cpp — a C++ host of the search path through include/gofann.h
// alone: loads a batch written by tests/test_batch_cpp.py (a manifest of
// named arrays and scalars), uploads it with the CUDA runtime, sizes and
// allocates the scratch, runs gofann_search_batch on one stream and writes
// the per-query top-k back as raw files.  It is the call sequence a C++
// integration of the reference's batch driver would make.
//
//   batch_driver <dir>    reads <dir>/manifest.txt and <dir>/<name>.bin,
//                         writes <dir>/out_ids.bin and <dir>/out_dists.bin
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <map>
#include <sstream>
#include <string>
#include <vector>

#include "gofann.h"

namespace {

struct Batch {
    std::string dir;
    std::map<std::string, void*> dev;
    std::map<std::string, size_t> bytes;
    std::map<std::string, double> scalar;
    std::vector<void*> owned;

    ~Batch()
    {
        for (void* p : owned) cudaFree(p);
    }
    bool load()
    {
        std::ifstream m(dir + "/manifest.txt");
        if (!m) return false;
        std::string kind, name;
        while (m >> kind >> name) {
            if (kind == "array") {
                size_t n = 0;
                m >> n;
                std::vector<char> host(n);
                std::ifstream f(dir + "/" + name + ".bin", std::ios::binary);
                if (!f.read(host.data(), static_cast<std::streamsize>(n))) return false;
                void* d = nullptr;
                if (cudaMalloc(&d, n > 0 ? n : 1) != cudaSuccess) return false;
                owned.push_back(d);
                if (n && cudaMemcpy(d, host.data(), n, cudaMemcpyHostToDevice) != cudaSuccess) return false;
                dev[name] = d;
                bytes[name] = n;
            } else {
                double v = 0;
                m >> v;
                scalar[name] = v;
            }
        }
        return true;
    }
    template <typename T>
    const T* a(const std::string& name) const
    {
        auto it = dev.find(name);
        return it == dev.end() ? nullptr : static_cast<const T*>(it->second);
    }
    double s(const std::string& name, double dflt = 0) const
    {
        auto it = scalar.find(name);
        return it == scalar.end() ? dflt : it->second;
    }
    uint32_t u(const std::string& name, double dflt = 0) const { return static_cast<uint32_t>(s(name, dflt)); }

    gofann_routes routes(const std::string& p) const
    {
        gofann_routes r{};
        r.n_routes = u(p + "n_routes");
        r.range_count = u(p + "range_count");
        r.query_row = a<uint32_t>(p + "query_row");
        r.group_id = a<uint32_t>(p + "group_id");
        r.start_local = a<uint32_t>(p + "start_local");
        r.filter_bits = a<uint64_t>(p + "filter_bits");
        r.range_modes = a<uint8_t>(p + "range_modes");
        r.range_lower = a<float>(p + "range_lower");
        r.range_upper = a<float>(p + "range_upper");
        r.qlabel_indptr = a<uint64_t>(p + "qlabel_indptr");
        r.qlabel_indices = a<uint32_t>(p + "qlabel_indices");
        r.primary_label = a<uint32_t>(p + "primary_label");
        r.pred_offsets = a<uint32_t>(p + "pred_offsets");
        r.clauses = a<gofann_clause>(p + "clauses");
        r.pred_handles = a<uint32_t>(p + "pred_handles");
        r.pred_ranges = a<gofann_range_atom>(p + "pred_ranges");
        r.pred_enabled = a<uint8_t>(p + "pred_enabled");
        r.route_compiled = a<uint8_t>(p + "route_compiled");
        return r;
    }
};

int die(const char* what, int st)
{
    std::fprintf(stderr, "%s failed (%d): %s\n", what, st, gofann_last_error());
    return 1;
}

}  // namespace

int main(int argc, char** argv)
{
    if (argc != 2) {
        std::fprintf(stderr, "usage: %s <batch dir>\n", argv[0]);
        return 2;
    }
    if (gofann_abi_version() != GOFANN_ABI_VERSION) {
        std::fprintf(stderr, "library ABI %d, header %d\n", gofann_abi_version(), GOFANN_ABI_VERSION);
        return 1;
    }
    Batch b;
    b.dir = argv[1];
    if (!b.load()) {
        std::fprintf(stderr, "cannot load %s\n", argv[1]);
        return 1;
    }

    gofann_index ix{};
    ix.graph.adjacency = b.a<uint32_t>("graph.adjacency");
    ix.graph.row_to_sample = b.a<uint32_t>("graph.row_to_sample");
    ix.graph.row_filter_mask = b.a<uint64_t>("graph.row_filter_mask");
    ix.graph.label_offset = b.a<uint32_t>("graph.label_offset");
    ix.graph.total_rows = b.u("graph.total_rows");
    ix.graph.degree = b.u("graph.degree");
    ix.graph.group_count = b.u("graph.group_count");
    ix.attrs.label_indptr = b.a<uint64_t>("attrs.label_indptr");
    ix.attrs.label_indices = b.a<uint32_t>("attrs.label_indices");
    ix.attrs.range_values = b.a<float>("attrs.range_values");
    ix.attrs.n_samples = b.u("attrs.n_samples");
    ix.attrs.range_count = b.u("attrs.range_count");
    ix.codes.pq_codes = b.a<uint8_t>("codes.pq_codes");
    ix.codes.pq_dim = b.u("codes.pq_dim");
    ix.codes.n_samples = b.u("attrs.n_samples");
    ix.codes.rq_codes = b.a<uint8_t>("codes.rq_codes");
    ix.codes.rq_factors = b.a<float>("codes.rq_factors");
    ix.codes.rq_anchor_ids = b.a<uint32_t>("codes.rq_anchor_ids");
    ix.codes.padded_dim = b.u("codes.padded_dim");
    ix.codes.num_anchors = b.u("codes.num_anchors");
    ix.pq_centroids = b.a<float>("pq_centroids");
    ix.base = b.a<void>("base");
    ix.base_dtype = static_cast<int32_t>(b.s("base_dtype"));
    ix.dim = b.u("dim");
    ix.posting_ids = b.a<uint32_t>("posting_ids");
    ix.rq_rotation = b.a<float>("rq_rotation");
    ix.rq_anchors = b.a<float>("rq_anchors");
    ix.rq_anchor_entry = b.a<uint32_t>("rq_anchor_entry");

    gofann_batch bt{};
    bt.queries = b.a<void>("queries");
    bt.n_queries = b.u("n_queries");
    bt.graph_routes = b.routes("g.");
    bt.posting_routes = b.routes("p.");
    bt.posting_begin = b.a<uint64_t>("posting_begin");
    bt.posting_count = b.a<uint32_t>("posting_count");
    bt.query_route_offsets = b.a<uint32_t>("query_route_offsets");
    bt.query_routes = b.a<uint32_t>("query_routes");

    gofann_batch_params p{};
    p.search.queue_size = static_cast<int32_t>(b.s("queue_size", 64));
    p.search.stop_width = static_cast<int32_t>(b.s("stop_width", 10));
    p.search.result_width = static_cast<int32_t>(b.s("result_width", 100));
    p.search.finish_limit = static_cast<int32_t>(b.s("finish_limit", 100));
    p.search.early_stop_mode = static_cast<int32_t>(b.s("early_stop_mode", GOFANN_EARLY_STOP_ADAPTIVE));
    p.search.max_steps = static_cast<int32_t>(b.s("max_steps", 0));
    p.search.scorer = static_cast<int32_t>(b.s("scorer", GOFANN_SCORER_PQ));
    p.search.predicate_bias = static_cast<int32_t>(b.s("predicate_bias", 1));
    p.search.alpha = static_cast<float>(b.s("alpha", 0.15));
    p.search.pq_mode = static_cast<int32_t>(b.s("pq_mode", GOFANN_PQ_LUT_GLOBAL));
    p.posting_shortlist = static_cast<int32_t>(b.s("posting_shortlist", 100));
    p.topk = static_cast<int32_t>(b.s("topk", 10));
    p.rq_entries = static_cast<int32_t>(b.s("rq_entries", 0));

    const size_t nbytes = gofann_search_batch_scratch_bytes(&ix, &bt, &p);
    if (nbytes == 0) return die("gofann_search_batch_scratch_bytes", 0);
    void* scratch = nullptr;
    uint32_t* ids = nullptr;
    float* dists = nullptr;
    int32_t* status = nullptr;
    const size_t out_n = static_cast<size_t>(bt.n_queries) * p.topk;
    if (cudaMalloc(&scratch, nbytes) != cudaSuccess || cudaMalloc(&ids, out_n * 4) != cudaSuccess ||
        cudaMalloc(&dists, out_n * 4) != cudaSuccess || cudaMalloc(&status, 4) != cudaSuccess ||
        cudaMemset(status, 0, 4) != cudaSuccess) {
        std::fprintf(stderr, "device allocation failed\n");
        return 1;
    }
    cudaStream_t stream;
    cudaStreamCreate(&stream);
    const int st = gofann_search_batch(&ix, &bt, &p, scratch, nbytes, ids, dists, status, stream);
    if (st != GOFANN_OK) return die("gofann_search_batch", st);
    if (cudaStreamSynchronize(stream) != cudaSuccess) {
        std::fprintf(stderr, "stream error: %s\n", cudaGetErrorString(cudaGetLastError()));
        return 1;
    }
    int32_t hst = 0;
    std::vector<uint32_t> hid(out_n);
    std::vector<float> hd(out_n);
    cudaMemcpy(&hst, status, 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(hid.data(), ids, out_n * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(hd.data(), dists, out_n * 4, cudaMemcpyDeviceToHost);
    std::ofstream(b.dir + "/out_ids.bin", std::ios::binary).write(reinterpret_cast<const char*>(hid.data()),
                                                                   static_cast<std::streamsize>(out_n * 4));
    std::ofstream(b.dir + "/out_dists.bin", std::ios::binary).write(reinterpret_cast<const char*>(hd.data()),
                                                                     static_cast<std::streamsize>(out_n * 4));
    cudaFree(scratch);
    cudaFree(ids);
    cudaFree(dists);
    cudaFree(status);
    cudaStreamDestroy(stream);
    std::printf("batch ok: %u queries, %u graph routes, %u posting routes, scratch %zu bytes, status %d\n",
                bt.n_queries, bt.graph_routes.n_routes, bt.posting_routes.n_routes, nbytes, hst);
    return hst == 0 ? 0 : 3;
}
