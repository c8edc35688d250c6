"""Configuration 4 end to end at a small scale on the GPU: FP16 512-d base,
64-byte 1-bit RaBitQ codes, degree-32 graph, tags, int64 ranges, exact and
fuzzy strings (the fuzzy rewrite runs the device's edit-distance check over
the string dictionary), hybrid AND, exact FP16 rerank.  The merged top-10
of every query must equal the CPU restatement of the same path (ids equal,
FP16 rerank distances within 1e-3 relative), and recall against the exact
filtered ground truth must be high."""
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import bench  # noqa: E402

pytestmark = pytest.mark.gpu


def test_config4_small_matches_oracle_and_recall():
    from gofann import workload_gpu as W, workload_hybrid as WH
    from gofann.rabitq_pipeline import RabitqPipeline
    torch.cuda.set_device(0)
    data = WH.generate(n=30_000, n_queries=400, n_strings=3000, n_centres=256, seed=3)
    idx = WH.build_index(data, seed=3)
    q = data["queries"]
    plan = WH.plan_queries(idx, data, q, scan_rows=2000)
    assert plan.graph_query.shape[0] > 0 and plan.posting_query.shape[0] > 0
    sel = np.arange(q.kind.shape[0])
    gt = WH.ground_truth(idx, data, q, plan, sel)
    # the fuzzy rewrite equals the oracle's edit distance over the dictionary
    from oracle import oracle as O
    dl, db = data["dict_len"], data["dict_bytes"]
    for i in np.nonzero(q.kind == 3)[0][:20]:
        want = [j for j in range(dl.shape[0])
                if abs(int(dl[j]) - len(q.string[i])) <= 2 and
                O.levenshtein(q.string[i], db[j, :dl[j]].tobytes()) <= 2]
        assert sorted(plan.matches[i].tolist()) == want
    pipe = RabitqPipeline(idx, plan, 96, shortlist=100)
    ids, d = pipe.run(q.vectors)
    torch.cuda.synchronize()
    gi, gd = ids.cpu().numpy().view(np.uint32), d.cpu().numpy()
    ci, cd = bench.c4_cpu_sample(idx, plan, q, pipe, sel, 96, 8)
    assert np.array_equal(gi, ci), f"ids differ for {int(np.any(gi != ci, axis=1).sum())} queries"
    ok = ci != bench.U32MAX
    assert np.all(np.abs(gd[ok] - cd[ok]) <= 1e-3 * np.maximum(np.abs(cd[ok]), 1e-30))
    rec = W.recall_at_k(gi, gt, 10)
    by = {nm: W.recall_at_k(gi[q.kind == k], gt[q.kind == k], 10) for k, nm in enumerate(WH.KIND_NAMES)}
    assert rec >= 0.9, (rec, by)
    assert by["exact_string"] >= 0.95 and by["fuzzy_string"] >= 0.95, by
