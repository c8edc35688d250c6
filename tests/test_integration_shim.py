"""The C++ shim of INTEGRATION.md compiles against include/gofann.h.

The shim is extracted from the document verbatim and compiled with g++
(-fsyntax-only) after mock declarations of the reference's contexts that
carry the reference's own field names and types (PqGraphSearchContext,
src/search/pq/backend_pq.cu:5930-6080; PqLowfreqSearchContext,
:10608-10630; PqSearchOptions, backend_pq.cuh:131-242; typedefs,
include/type_def.h).  A renamed field or a changed ABI signature fails the
compile.
"""
import re
import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]

MOCKS = r'''
#include <cstddef>
#include <cstdint>
#include <memory>
typedef void* cudaStream_t;
typedef uint8_t pq_idx_t;   // include/type_def.h
typedef float pq_value_t;
typedef uint8_t value_t;
typedef uint64_t idx_t;
[[noreturn]] void fail_pq(const char* message);
struct PqSearchOptions {
    float predicate_bias_alpha = 0.0f;
    int dim = 128;
    int pq_dim = 64;
    int topk = 10;
    int search_queue_size = 50;
    int search_finish_count = 1;
};
struct PqPredicateDeviceState { bool bias_frontier = false; };
struct PqGraphSearchContext {
    uint32_t stop_width = 10;
    uint32_t result_width = 10;
    uint32_t resident_base_rows = 0;
    const pq_idx_t* d_data = nullptr;
    value_t* d_query = nullptr;
    idx_t* d_result = nullptr;
    float* d_result_dist = nullptr;
    const pq_value_t* d_pq_centroid = nullptr;
    pq_value_t* d_pq_table = nullptr;
    uint32_t* d_query_group_ids = nullptr;
    uint32_t* d_start_local_ids = nullptr;
    uint32_t* d_row_to_sample = nullptr;
    uint32_t* d_label_offset = nullptr;
    uint64_t* d_row_filter_mask = nullptr;
    uint64_t* d_query_filter_bits = nullptr;
    uint8_t* d_query_range_modes = nullptr;
    float* d_query_range_lower_bounds = nullptr;
    float* d_query_range_upper_bounds = nullptr;
    float* d_base_range_values = nullptr;
    uint32_t* d_resident_graph = nullptr;
    uint8_t* d_resident_base_vectors = nullptr;
    uint64_t* d_resident_data_label_indptr = nullptr;
    uint32_t* d_resident_data_label_indices = nullptr;
    uint64_t* d_resident_query_label_indptr = nullptr;
    uint32_t* d_resident_query_label_indices = nullptr;
    uint32_t* d_resident_query_filter_labels = nullptr;
    std::unique_ptr<PqPredicateDeviceState> predicate;
};
struct PqLowfreqSearchContext {
    const pq_idx_t* d_data = nullptr;
    const pq_value_t* d_pq_centroid = nullptr;
    const value_t* d_all_query = nullptr;
    idx_t* d_result = nullptr;
    float* d_result_dist = nullptr;
    pq_value_t* d_pq_table = nullptr;
    uint32_t* d_candidate_ids = nullptr;
    uint32_t* d_candidate_offsets = nullptr;
    uint32_t* d_candidate_sizes = nullptr;
};
'''


def test_integration_shim_compiles(tmp_path):
    text = (ROOT / "INTEGRATION.md").read_text()
    blocks = re.findall(r"```cpp\n(.*?)```", text, re.S)
    assert blocks, "no C++ block in INTEGRATION.md"
    src = tmp_path / "shim.cpp"
    src.write_text(MOCKS + "\n".join(blocks))
    r = subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-Wall", "-Wextra", "-Wno-unused-function",
                        "-I", str(ROOT / "include"), str(src)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]
