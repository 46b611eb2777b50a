"""Host logic of nekochat_b200.generate (the engine's prefix reuse and prefill chunking, engine.cpp:74-112)."""
import numpy as np

from nekochat_b200.generate import common_prefix, fit_prompt, prefill_chunks


def test_common_prefix_keeps_one_token_to_rerun():
    assert common_prefix([], [5, 6, 7]) == 0
    assert common_prefix([5, 6, 9], [5, 6, 7]) == 2
    assert common_prefix([5, 6, 7], [5, 6, 7]) == 2        # identical prompt: the last token is re-run
    assert common_prefix([5, 6, 7, 8], [5, 6]) == 1        # shorter prompt inside the cache
    assert common_prefix([5], [5, 6, 7]) == 1
    assert common_prefix([1], [2]) == 0


def test_fit_prompt_empty_and_overlong():
    assert fit_prompt([], 16, eos=3) == [3]
    assert fit_prompt(list(range(20)), 16) == list(range(5, 20))   # context - 1 last tokens
    assert fit_prompt(list(range(15)), 16) == list(range(15))


def test_prefill_chunks_end_before_the_last_token():
    assert prefill_chunks(0, 10, 64) == [(0, 9), (9, 10)]
    assert prefill_chunks(0, 130, 64) == [(0, 64), (64, 128), (128, 129), (129, 130)]
    assert prefill_chunks(0, 65, 64) == [(0, 64), (64, 65)]
    assert prefill_chunks(7, 8, 64) == [(7, 8)]
    assert prefill_chunks(0, 1, 64) == [(0, 1)]


class FakeRunner:
    """A deterministic stand-in for nekochat_b200.model.Model with the device loop's contract (neko_model_stage,
    neko_model_step, neko_model_set_stop, neko_model_generated as include/neko_cuda.h states it): the greedy token
    after token t at position p is (7 t + p) % V, so host and device phases can be compared exactly on CPU."""

    def __init__(self, context, V=50):
        self.cfg = type("cfg", (), {"context": context, "max_rows": 16})
        self.V = V
        self.kv = {}  # (slot, pos) -> token run there

    def nxt(self, t, p):
        return (7 * t + p) % self.V

    def forward(self, tokens, pos0, slot=0):
        for j, t in enumerate(tokens):
            assert pos0 + j < self.cfg.context
            self.kv[(slot, pos0 + j)] = int(t)
        out = np.zeros(self.V, np.float32)
        out[self.nxt(int(tokens[-1]), pos0 + len(tokens) - 1)] = 1.0
        return out

    def set_stop(self, ids, max_new):
        self.stops, self.max_new = set(ids), max_new

    def stage(self, slots, tokens, pos):
        self.slots, self.tok, self.pos = list(slots), list(tokens), list(pos)
        self.log = [[] if t in self.stops else [t] for t in tokens]
        self.state = [1 if t in self.stops else (0 if self.max_new <= 1 else -1) for t in tokens]
        self.frozen = list(zip(tokens, pos))

    def step(self, n, max_pos):
        for i in range(n):
            assert self.pos[i] <= max_pos and self.pos[i] + 1 < self.cfg.context
            self.kv[(self.slots[i], self.pos[i])] = self.tok[i]
            t, p = self.nxt(self.tok[i], self.pos[i]), self.pos[i] + 1
            if self.state[i] >= 0:
                self.tok[i], self.pos[i] = self.frozen[i]
                continue
            self.tok[i], self.pos[i] = t, p
            if t in self.stops:
                self.state[i], self.frozen[i] = 1, (t, p)
                continue
            self.log[i].append(t)
            if len(self.log[i]) == self.max_new:
                self.state[i], self.frozen[i] = 0, (t, p)

    def generated(self, n):
        return [np.array(self.log[i], np.int32) for i in range(n)], np.array(self.state[:n], np.int32)


def test_batch_generator_host_logic_matches_slot_generator():
    """BatchGenerator (device phase + host finish) == SlotGenerator (the engine's loop, one token per forward)
    per slot, over turns with prefix reuse, stop ids, max_new and the context limit."""
    from nekochat_b200.generate import BatchGenerator, SlotGenerator
    rng = np.random.default_rng(2)
    for trial in range(30):
        ctx = int(rng.integers(8, 40))
        stops = [int(t) for t in rng.integers(0, 50, int(rng.integers(0, 3)))]
        fb, fs = FakeRunner(ctx), FakeRunner(ctx)
        bg = BatchGenerator(fb, stop_ids=stops)
        sg = {s: SlotGenerator(fs, slot=s, stop_ids=stops) for s in range(3)}
        hist = {s: [] for s in range(3)}
        for turn in range(3):
            prompts = {s: hist[s] + [int(t) for t in rng.integers(0, 50, int(rng.integers(1, ctx + 4)))]
                       for s in range(3)}
            max_new = int(rng.integers(1, 15))
            got = bg.generate(prompts, max_new)
            for s in range(3):
                want, st = sg[s].generate(prompts[s], max_new)
                assert got[s][0] == want, (trial, turn, s)
                for k in ("stop_reason", "reused_tokens", "generated_tokens", "prompt_tokens"):
                    assert got[s][1][k] == st[k], (trial, turn, s, k)
                assert bg.cached[s] == sg[s].cached
                hist[s] = prompts[s] + want
