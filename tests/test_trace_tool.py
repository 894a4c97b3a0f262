"""The step-timeline summary of diolkos_b200.trace on a synthetic stamp array (CPU, no GPU)."""
import numpy as np

from diolkos_b200 import trace as T


def _stamps(n_layers=2, grid=3):
    """Ops 1000 ns apart: with b = 1000 (i + 1), op i's input is seen at b + 10 + cta, ready at b + 50,
    its activation built at b + 150 and the op finished at b + 600 + 10 * cta."""
    O = 5 * n_layers + 1
    tr = np.zeros((grid, O, T.SLOTS), np.int64)
    for i in range(O):
        for c in range(grid):
            base = 1000 * (i + 1)
            tr[c, i, T.SEEN] = base + 10 + c
            tr[c, i, T.READY] = base + 50
            tr[c, i, T.ACT] = base + 150
            tr[c, i, T.FIN] = base + 600 + 10 * c
    return tr


def test_summary_of_synthetic_stamps():
    tr = _stamps()
    res = T.summarise(tr)
    assert [len(res[k]["span"]) for k in T.KINDS] == [2] * 5 and len(res["cls"]["span"]) == 1
    # act: ready -> activation, 100 ns; cons: activation -> finish, 450 + 10 * cta ns, median 460 ns
    for k in T.KINDS + ["cls"]:
        assert np.allclose(res[k]["act"], 0.1) and np.allclose(res[k]["cons"], 0.46)
    # seen: the first CTA's sight of the input after the previous op's last CTA (1000 + 10 - 620 ns)
    assert np.allclose(res["attn"]["seen"], 0.39) and res["qkv"]["seen"][0] == 0.0
    # span: previous op's last finish -> this op's last finish, 1000 ns (the first op: from its ready)
    assert np.allclose(res["wo"]["span"], 1.0) and np.isclose(res["qkv"]["span"][0], 0.57)


def test_ops_that_did_not_run_are_skipped():
    tr = _stamps()
    tr[:, 3, T.FIN] = 0  # op 3 recorded nothing
    res = T.summarise(tr)
    assert len(res["w13"]["span"]) == 1
    assert np.isclose(res["w2"]["span"][0], 2.0)  # measured from op 2's end
