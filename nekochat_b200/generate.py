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


class BatchGenerator:
    """Engine::generate for several slots at once. Each slot's prompt runs with the engine's prefix reuse and
    prefill chunking (as SlotGenerator); then every slot decodes together on the device: neko_model_stage +
    neko_model_step with the stop ids and token budget of neko_model_set_stop, with no per-token host round trip.
    The device phase stops one position short of the smallest remaining context (a step cannot advance past the
    last position); slots still running then finish on the host one token per forward, with the engine's
    context-full stop (reason 3)."""

    def __init__(self, model, stop_ids=(), eos=0):
        self.m = model
        self.stop_ids = [int(t) for t in stop_ids]
        self.eos = eos
        self.cached = {}  # slot -> the tokens its KV cache holds

    def generate(self, prompts, max_new):
        """prompts: {slot: token list}. Returns {slot: (generated tokens, stats dict as SlotGenerator's)}."""
        ctx = self.m.cfg.context
        slots = sorted(prompts)
        firsts, pos, stats = [], [], {}
        for slot in slots:
            prompt = fit_prompt(prompts[slot], ctx, self.eos)
            common = common_prefix(self.cached.get(slot, []), prompt)
            cached = self.cached.get(slot, [])[:common]
            for b, e in prefill_chunks(common, len(prompt), min(MAX_BATCH, self.m.cfg.max_rows)):
                logits = self.m.forward(np.asarray(prompt[b:e], np.int32), len(cached), slot)
                cached.extend(prompt[b:e])
            self.cached[slot] = cached
            firsts.append(int(np.argmax(logits)))
            pos.append(len(cached))
            stats[slot] = {"prompt_tokens": len(prompt), "reused_tokens": common}
        if max_new <= 0:
            return {s: ([], dict(stats[s], generated_tokens=0, stop_reason=0)) for s in slots}
        n = len(slots)
        steps = max(0, min(max_new - 1, min(ctx - 1 - p for p in pos)))
        self.m.set_stop(self.stop_ids, max_new)
        self.m.stage(slots, firsts, pos)
        for k in range(steps):
            self.m.step(n, max(pos) + k)
        outs, reasons = self.m.generated(n)
        self.m.set_stop([], 0)
        result = {}
        for i, slot in enumerate(slots):
            out, why = [int(t) for t in outs[i]], int(reasons[i])
            cached = self.cached[slot]
            if why == 1:
                cached.extend(out)          # every logged token was run
            elif why == 0:
                cached.extend(out[:-1])     # the last one never runs
            else:                           # running: all but the last logged token were run on the device
                cached.extend(out[:-1])
                why = self._finish(slot, out, cached, max_new, ctx)
            result[slot] = (out, dict(stats[slot], generated_tokens=len(out), stop_reason=why))
        return result

    def _finish(self, slot, out, cached, max_new, ctx):
        """The rest of the engine's loop (engine.cpp:122-137) for one slot whose last token is not yet run."""
        stops = set(self.stop_ids)
        while True:
            if len(cached) >= ctx:
                return 3
            if len(out) == max_new:
                return 0
            logits = self.m.forward(np.array([out[-1]], np.int32), len(cached), slot)
            cached.append(out[-1])
            nxt = int(np.argmax(logits))
            if nxt in stops:
                return 1
            out.append(nxt)
