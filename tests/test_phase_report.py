"""The phase report's aggregation of profiled stamps (CFB_BUF_PROF), on a hand-made record."""
import torch

from chain_flow_b200.phase_report import summarize


def test_summarize_wall_and_barrier_tail():
    P, G = 3, 2
    t = torch.zeros(P, G, 20, dtype=torch.int64)
    # phase 0 starts at 1000 ns; CTA 1 finishes its work last (3000), its epilogue at 3500, and
    # the last CTA passes the barrier at 4500
    t[0, :, 0] = torch.tensor([1000, 1200])
    t[0, :, 1] = torch.tensor([2000, 3000])
    t[0, :, 6] = torch.tensor([2500, 3500])
    t[0, :, 2] = torch.tensor([4400, 4500])
    # phase 1: a non-GEMM phase, which writes no epilogue stamp: its slot 6 holds whatever an
    # earlier run left there (here a stale value far outside the run); work done at 6000,
    # barrier passed at 7000
    t[1, :, 1] = torch.tensor([6000, 5500])
    t[1, :, 6] = torch.tensor([-(1 << 62), 1 << 62])
    t[1, :, 2] = torch.tensor([7000, 6900])
    # phase 2: same class as phase 0
    t[2, :, 1] = torch.tensor([9000, 8000])
    t[2, :, 6] = torch.tensor([9500, 9100])
    t[2, :, 2] = torch.tensor([10500, 10400])
    tab = torch.zeros(P, 15, dtype=torch.int32)
    tab[0, 0], tab[0, 3], tab[0, 4], tab[0, 5] = 1, 600, 20, 0
    tab[1, 0] = 2
    tab[2, 0], tab[2, 3], tab[2, 4], tab[2, 5] = 1, 600, 20, 0
    s = summarize(t, tab)
    assert abs(s["total_us"] - 9.5) < 1e-9
    walls = [r["wall_us"] for r in s["phases"]]
    assert walls == [3.5, 2.5, 3.5]
    tails = [r["tail_us"] for r in s["phases"]]
    assert tails == [1.0, 1.0, 1.0]
    c = s["classes"][(1, 600, 20)]
    assert c["n"] == 2 and abs(c["wall_us"] - 7.0) < 1e-9 and abs(c["tail_us"] - 2.0) < 1e-9
    assert s["classes"][(2, 0, 0)]["n"] == 1
    assert sum(v["n"] for v in s["classes"].values()) == P
