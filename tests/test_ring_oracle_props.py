"""Size-independent properties of the context-ring oracle (CPU): after any sequence of chain
writes, a gather returns the last C rows written (oldest first), front-padded with the oldest row
while fewer than C are valid; a masked-off request changes nothing but the trash row."""
import torch

from oracle.ring import ring_gather, ring_write

C, H, KMAX = 5, 3, 3


def _window(stream):
    last = stream[-C:]
    return [last[0]] * (C - len(last)) + last


def test_gather_is_the_last_rows_written():
    slots = 2
    ring = torch.zeros(slots, C + 1, H, dtype=torch.float16)
    rpos = torch.zeros(slots, dtype=torch.long)
    nval = torch.zeros(slots, dtype=torch.long)
    streams = {0: [], 1: []}
    counts = [1, 3, 2, 3, 1, 2, 3, 3]
    nxt = 1
    for step, cnt0 in enumerate(counts):
        cnt = torch.tensor([cnt0, KMAX - cnt0 + 1])
        rows = torch.tensor([0, 1])
        # each request's accepted rows are consecutive rows of sh starting at starts[b]
        sh = torch.arange(nxt, nxt + 2 * KMAX, dtype=torch.float32)[:, None].repeat(1, H)
        starts = torch.tensor([0, KMAX])
        ring_write(ring, rpos, nval, sh, rows, starts, cnt, torch.tensor([True, True]), None, KMAX)
        for b in range(2):
            streams[b] += [float(sh[int(starts[b]) + j, 0]) for j in range(int(cnt[b]))]
        nxt += 2 * KMAX
        got = ring_gather(ring, rpos, nval, rows)
        for b in range(2):
            assert got[b, :, 0].tolist() == _window(streams[b]), (step, b)
            assert int(nval[b]) == min(len(streams[b]), C)


def test_masked_request_keeps_its_window():
    ring = torch.zeros(1, C + 1, H, dtype=torch.float16)
    rpos = torch.zeros(1, dtype=torch.long)
    nval = torch.zeros(1, dtype=torch.long)
    rows = torch.tensor([0])
    sh = torch.arange(1, 1 + KMAX, dtype=torch.float32)[:, None].repeat(1, H)
    ring_write(ring, rpos, nval, sh, rows, torch.tensor([0]), torch.tensor([2]), torch.tensor([True]), None, KMAX)
    before = (ring[0, :C].clone(), int(rpos[0]), int(nval[0]))
    ring_write(ring, rpos, nval, sh + 100, rows, torch.tensor([0]), torch.tensor([3]), torch.tensor([False]),
               None, KMAX)
    assert torch.equal(ring[0, :C], before[0])
    assert (int(rpos[0]), int(nval[0])) == before[1:]
    assert ring_gather(ring, rpos, nval, rows)[0, :, 0].tolist() == [1.0, 1.0, 1.0, 1.0, 2.0]
