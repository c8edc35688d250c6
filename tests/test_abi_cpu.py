"""C-ABI checks that need no GPU: the library loads, exports every symbol
include/gofann.h declares, and the ctypes mirror matches the C layouts."""
import ctypes as C
import subprocess
import tempfile
from pathlib import Path

import pytest

from gofann import _abi as A

ROOT = Path(__file__).resolve().parents[1]


def test_library_exports_every_header_symbol():
    declared = A.header_symbols()
    assert len(declared) >= 16
    lib = A.lib()
    for name in declared:
        assert hasattr(lib, name), name
    assert set(declared) == set(A.EXPORTED)
    assert lib.gofann_abi_version() == 4


def test_nm_dynamic_symbols():
    out = subprocess.run(["nm", "-D", "--defined-only", str(A.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    for name in A.header_symbols():
        assert name in exported, name


def test_struct_layouts_match_c():
    src = r'''
#include <stdio.h>
#include <stddef.h>
#include "gofann.h"
#define S(T) printf(#T " %zu\n", sizeof(T));
#define O(T, f) printf(#T "." #f " %zu\n", offsetof(T, f));
int main(void) {
  S(gofann_clause) S(gofann_range_atom) S(gofann_graph) S(gofann_attrs) S(gofann_codes)
  S(gofann_prepared) S(gofann_routes) S(gofann_search_params) S(gofann_search_out)
  S(gofann_index) S(gofann_batch) S(gofann_batch_params)
  O(gofann_index, pq_centroids) O(gofann_index, base_dtype) O(gofann_index, rq_anchor_entry)
  O(gofann_batch, graph_routes) O(gofann_batch, posting_routes) O(gofann_batch, query_routes)
  O(gofann_batch_params, posting_shortlist) O(gofann_batch_params, rq_entries)
  O(gofann_codes, rq_codes) O(gofann_codes, padded_dim) O(gofann_routes, query_row)
  O(gofann_routes, route_compiled) O(gofann_search_params, alpha) O(gofann_search_params, pq_mode) O(gofann_search_params, resident_warps) O(gofann_prepared, dim) O(gofann_prepared, pq_query)
  O(gofann_graph, total_rows) O(gofann_graph, records) O(gofann_graph, record_stride) O(gofann_attrs, n_samples) O(gofann_prepared, n_rows)
  return 0; }
'''
    with tempfile.TemporaryDirectory() as d:
        c = Path(d) / "l.c"
        c.write_text(src)
        exe = Path(d) / "l"
        subprocess.run(["gcc", "-I", str(ROOT / "include"), str(c), "-o", str(exe)], check=True)
        lines = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    got = dict(ln.split() for ln in lines if ln)
    py = {"gofann_clause": A.Clause, "gofann_range_atom": A.RangeAtom, "gofann_graph": A.Graph,
          "gofann_attrs": A.Attrs, "gofann_codes": A.Codes, "gofann_prepared": A.Prepared,
          "gofann_routes": A.Routes, "gofann_search_params": A.SearchParams, "gofann_search_out": A.SearchOut,
          "gofann_index": A.Index, "gofann_batch": A.Batch, "gofann_batch_params": A.BatchParams}
    for cname, st in py.items():
        assert int(got[cname]) == C.sizeof(st), cname
    for key, val in got.items():
        if "." in key:
            t, f = key.split(".")
            assert getattr(py[t], f).offset == int(val), key
    assert A.CLAUSE_DTYPE.itemsize == C.sizeof(A.Clause)
    assert A.RANGE_ATOM_DTYPE.itemsize == C.sizeof(A.RangeAtom)


def test_invalid_arguments_rejected_without_gpu():
    """Argument validation runs before any CUDA call and reports a message."""
    lib = A.lib()
    st = lib.gofann_pq_build_lut(None, 0, 1, 128, None, 32, None, None)
    assert st == A.ERR_INVALID
    assert b"null" in lib.gofann_last_error()
    st = lib.gofann_rerank(C.c_void_p(8), 0, 10, 8, C.c_void_p(8), None, C.byref(A.Routes()), C.c_void_p(8), 10, 11,
                           C.c_void_p(8), C.c_void_p(8), None)
    assert st == A.ERR_INVALID
    p = A.fill_params(queue_size=1)
    g, at, cs, pr, rs, out = A.Graph(), A.Attrs(), A.Codes(), A.Prepared(), A.Routes(), A.SearchOut()
    st = lib.gofann_beam_search(C.byref(g), C.byref(at), C.byref(cs), C.byref(pr), C.byref(rs), C.byref(p),
                                C.byref(out), C.c_void_p(8), 0, None)
    assert st == A.ERR_INVALID and b"queue_size" in lib.gofann_last_error()
    st = lib.gofann_shard_merge(C.c_void_p(8), C.c_void_p(8), 0, 4, 10, C.c_void_p(8), C.c_void_p(8), None)
    assert st == A.ERR_INVALID
