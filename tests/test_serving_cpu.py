"""The continuous batcher's bookkeeping on CPU, with a stand-in model: next token = last + 1.
Requests join when a row and blocks are free, leave when done, the live rows stay packed at
0..n-1 (finished rows refilled by moving the last one), positions equal the rows already cached,
and every block returns to the pools."""
import pytest

torch = pytest.importorskip("torch")

from mllm_b200 import runtime as rt  # noqa: E402
from mllm_b200.serving import ContinuousBatcher  # noqa: E402


class CountingModel:
    vocab = 1000

    def __init__(self):
        self.calls = []

    def new_caches(self, num_blocks, block_size, max_seqs, max_blocks_per_seq):
        return [rt.PagedKVCache(num_blocks, 1, 8, block_size, max_seqs, max_blocks_per_seq, device="cpu")
                for _ in range(2)]

    def forward(self, ids, positions, caches):
        B, S = ids.shape
        before = caches[0].host_lengths()[:B]
        if S == 1:
            assert positions.tolist() == before          # the new token's position = rows cached
        else:
            assert B == 1 and positions.tolist() == list(range(before[0], before[0] + S))
        for c in caches:
            c.advance(S, batch=B)
        self.calls.append((B, S))
        logits = torch.zeros(B, self.vocab)
        logits[torch.arange(B), (ids[:, -1] + 1) % self.vocab] = 1.0
        return logits


def test_requests_join_and_leave_between_steps():
    m = CountingModel()
    bat = ContinuousBatcher(m, max_batch=2, num_blocks=6, block_size=128)
    specs = [([5, 6, 7], 4), ([100] * 200, 3), ([40], 6), ([9] * 129, 2), ([1, 2], 1)]
    ids = [bat.submit(p, n) for p, n in specs]
    seen_live = set()
    while bat.waiting or bat.live:
        bat.step()
        n = len(bat.live)
        seen_live.add(n)
        assert n <= 2
        lens = bat.caches[0].host_lengths()
        for i, r in enumerate(bat.live):      # row i holds live[i]: prompt + tokens fed so far
            assert lens[i] == len(r.prompt) + len(r.tokens) - 1
        assert all(x == 0 for x in lens[n:])
    out = {rid: r.tokens for rid, r in bat.done.items()}
    for rid, (p, n) in zip(ids, specs):
        assert out[rid] == [(p[-1] + k) % m.vocab for k in range(1, n + 1)]
    for c in bat.caches:
        assert c.free_blocks == 6 and c.host_lengths() == [0, 0]
    assert 2 in seen_live                       # requests really ran side by side
    # the 200-token prompt needs 2 blocks per layer for 203 rows; with 6 blocks at most two
    # such requests fit, so admission waited for blocks at some point
    assert max(b for b, s in m.calls if s == 1) == 2


def test_a_request_that_can_never_fit_is_refused():
    bat = ContinuousBatcher(CountingModel(), max_batch=2, num_blocks=2, block_size=128)
    with pytest.raises(ValueError):
        bat.submit([1] * 300, 10)              # 310 rows need 3 blocks, the pool has 2


def test_move_keeps_block_ownership():
    c = rt.PagedKVCache(8, 1, 8, 128, max_seqs=3, device="cpu")
    c.set_lengths([130, 5, 260])
    blocks2 = c.blocks_of(2)
    c.release(0)
    c.move(2, 0)
    assert c.blocks_of(0) == blocks2 and c.blocks_of(2) == []
    assert c.host_lengths() == [260, 5, 0]
    assert c.lengths.tolist() == [260, 5, 0]
    assert c.block_table[0, :3].tolist() == blocks2
    with pytest.raises(RuntimeError):
        c.move(1, 0)                            # row 0 is occupied
    v = c.slot(1)
    v.advance(3)
    assert c.host_lengths()[1] == 8 and v.length_of(1) == 8


class PackedCountingModel(CountingModel):
    """Also takes several prompts in one pass (forward_packed), as DecoderModel does."""

    def forward_packed(self, ids, q_lens, caches):
        v = caches[0]
        assert len(v.host_lengths()) == len(q_lens) and all(n == 0 for n in v.host_lengths())
        assert ids.numel() == sum(q_lens)
        for c in caches:
            c.advance(list(q_lens), batch=len(q_lens))
        self.calls.append(("packed", tuple(q_lens)))
        last = torch.tensor([sum(q_lens[:b + 1]) - 1 for b in range(len(q_lens))])
        logits = torch.zeros(len(q_lens), self.vocab)
        logits[torch.arange(len(q_lens)), (ids[last] + 1) % self.vocab] = 1.0
        return logits


def test_joining_prompts_are_prefilled_together():
    m = PackedCountingModel()
    bat = ContinuousBatcher(m, max_batch=3, num_blocks=8, block_size=128)
    specs = [([5, 6, 7], 4), ([100] * 200, 3), ([40], 6), ([9] * 129, 2), ([1, 2], 1)]
    ids = [bat.submit(p, n) for p, n in specs]
    while bat.waiting or bat.live:
        bat.step()
        lens = bat.caches[0].host_lengths()
        for i, r in enumerate(bat.live):
            assert lens[i] == len(r.prompt) + len(r.tokens) - 1
    out = {rid: r.tokens for rid, r in bat.done.items()}
    for rid, (p, n) in zip(ids, specs):
        assert out[rid] == [(p[-1] + k) % m.vocab for k in range(1, n + 1)]
    packed = [c[1] for c in m.calls if c[0] == "packed"]
    assert packed[0] == (3, 200, 1)              # the first three prompts in one pass
    assert sum(len(p) for p in packed) == len(specs)
    for c in bat.caches:
        assert c.free_blocks == 8 and all(x == 0 for x in c.host_lengths())


def test_slot_view_of_several_rows():
    c = rt.PagedKVCache(8, 1, 8, 128, max_seqs=4, device="cpu")
    c.set_lengths([10, 0, 0, 0])
    v = c.slot(1, 2)
    v.advance([130, 5], batch=2)
    assert c.host_lengths() == [10, 130, 5, 0] and c.lengths.tolist() == [10, 130, 5, 0]
    assert v.host_lengths() == [130, 5] and v.lengths.tolist() == [130, 5]
    assert len(c.blocks_of(1)) == 2 and len(v.blocks_of(1)) == 1
    assert v.block_table.shape[0] == 2 and v.block_table[0, :2].tolist() == c.blocks_of(1)
    with pytest.raises(RuntimeError):
        v.reserve(2, 1)                          # outside the view
    with pytest.raises(RuntimeError):
        c.slot(3, 2)                             # past the parent's rows
    v.release(0)
    assert c.host_lengths() == [10, 0, 5, 0] and c.free_blocks == 8 - 2


def test_decode_graph_policy(monkeypatch):
    """When the batcher records a decode graph (a batch size seen two steps running), reuses it
    (same size, rows within its bound), records again (a longer request joined) or evicts one
    (more sizes than max_graphs).  The graph class is a stand-in: this runs on CPU."""
    from mllm_b200 import serving

    made = []

    class FakeGraph:
        def __init__(self, model, caches, n, max_len):
            self.n, self.max_len = n, max_len
            made.append((n, max_len))

        def replay(self, ids, pos):
            for c in bat.caches:                 # the recorded step advances the device lengths
                c.lengths[:self.n] += 1
            return bat.model.forward_logits(ids)

    class Model(CountingModel):
        def forward_logits(self, ids):
            B = ids.shape[0]
            logits = torch.zeros(B, self.vocab)
            logits[torch.arange(B), (ids[:, -1] + 1) % self.vocab] = 1.0
            return logits

    monkeypatch.setattr(serving, "DecodeGraph", FakeGraph)
    bat = ContinuousBatcher(Model(), max_batch=2, num_blocks=12, block_size=128, graphs=False, max_graphs=1)
    bat.graphs = True                            # as on a GPU model
    a = bat.submit([1] * 10, 6)
    bat.step()                                   # admission + an eager step (first time n = 1)
    assert made == [] and bat.graph_steps == 0
    bat.step()                                   # n = 1 again: recorded and replayed
    assert made == [(1, 256)] and bat.graph_steps == 1
    bat.step()
    assert made == [(1, 256)] and bat.graph_steps == 2
    b = bat.submit([2] * 300, 3)                 # joins: n = 2, 303 rows -> bound 512
    bat.step()
    assert len(made) == 1                        # a new size: eager this step
    bat.step()
    assert made[-1] == (2, 512) and list(bat._graphs) == [2]   # max_graphs = 1: the n = 1 graph is gone
    out = bat.run()
    assert out[a] == [(1 + k) % 1000 for k in range(1, 7)] and out[b] == [3, 4, 5]
    for c in bat.caches:
        assert c.host_lengths() == [0] * 2 and c.lengths.tolist() == [0, 0] and c.free_blocks == 12
