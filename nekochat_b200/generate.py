"""Chat-turn generation on the native runner with the engine's semantics (Engine::generate, engine.cpp:74-142):
the KV cache of a slot is reused for the longest common prefix of the new prompt and the tokens the slot already
holds (at least one prompt token is re-run, for fresh logits), the rest of the prompt runs in chunks of at most 64
tokens (Model::kMaxBatch, model.h:66) that end one token before the prompt's end (the engine's restore point),
then greedy decoding (Sampler::sample at temperature 0, sampler.cpp:24: the first index of the maximum) stops at
a stop id, at max_new tokens, or when the context is full.

Stop reasons follow GenerateStats::stopReason: 0 max_new reached, 1 stop id, 3 context full.
"""
import numpy as np

MAX_BATCH = 64  # Model::kMaxBatch


def common_prefix(cached, prompt):
    """Tokens of `cached` that the new prompt can keep (engine.cpp:86-89): the longest common prefix, but never the
    whole prompt, so at least one prompt token is re-run."""
    n = 0
    while n < len(cached) and n < len(prompt) and cached[n] == prompt[n]:
        n += 1
    if n == len(prompt):
        n -= 1
    return max(n, 0)


def fit_prompt(prompt, context, eos=0):
    """The prompt the engine runs (engine.cpp:81-83): an empty prompt becomes [eos], one of context tokens or more
    keeps its last context - 1."""
    p = [int(t) for t in prompt]
    if not p:
        p = [eos]
    if len(p) >= context:
        p = p[len(p) - (context - 1):]
    return p


def prefill_chunks(start, end, max_batch):
    """[begin, end) token ranges of the prompt run (engine.cpp:98-112): at most max_batch each, and a chunk that
    would cross the last prompt token ends just before it."""
    restore_at = end - 1
    out, i = [], start
    while i < end:
        e = min(end, i + max_batch)
        if i < restore_at < e:
            e = restore_at
        out.append((i, e))
        i = e
    return out


class SlotGenerator:
    """Generation for one slot of a nekochat_b200.model.Model, keeping the tokens its KV cache holds."""

    def __init__(self, model, slot=0, stop_ids=(), eos=0):
        self.m = model
        self.slot = slot
        self.stop_ids = set(int(t) for t in stop_ids)
        self.eos = eos
        self.cached = []

    def generate(self, prompt, max_new, keep_logits=False):
        """Returns (generated tokens, stats dict: prompt_tokens, reused_tokens, generated_tokens, stop_reason,
        and, with keep_logits, the logits each sampled token was taken from)."""
        ctx = self.m.cfg.context
        prompt = fit_prompt(prompt, ctx, self.eos)
        common = common_prefix(self.cached, prompt)
        self.cached = self.cached[:common]
        stats = {"prompt_tokens": len(prompt), "reused_tokens": common, "generated_tokens": 0, "stop_reason": 0}
        logits = None
        for b, e in prefill_chunks(common, len(prompt), min(MAX_BATCH, self.m.cfg.max_rows)):
            logits = self.m.forward(np.asarray(prompt[b:e], np.int32), len(self.cached), self.slot)
            self.cached.extend(prompt[b:e])
        out, seen = [], []
        for n in range(max_new):
            nxt = int(np.argmax(logits))
            if keep_logits:
                seen.append(logits)
            if nxt in self.stop_ids:
                stats["stop_reason"] = 1
                break
            out.append(nxt)
            stats["generated_tokens"] += 1
            if len(self.cached) >= ctx:
                stats["stop_reason"] = 3
                break
            if n + 1 == max_new:  # no model run for a token that will not be sampled
                break
            logits = self.m.forward(np.array([nxt], np.int32), len(self.cached), self.slot)
            self.cached.append(nxt)
        if keep_logits:
            stats["logits"] = seen
        return out, stats
