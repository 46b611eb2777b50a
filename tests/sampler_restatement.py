"""numpy restatement of Sampler::sample (sampler.cpp:14-55) with the uniform draw as an input, for the sampler
tests (test infrastructure): the reference's token for a seed equals this with u = the seed's draw, and the
device sampler is checked against the reference itself."""
import numpy as np


def penalize(logits, history, repeat_penalty, repeat_last_n):
    x = np.array(logits, dtype=np.float32)
    if repeat_penalty != 1.0 and repeat_last_n > 0:
        seen = set()
        h = list(history)[max(0, len(history) - repeat_last_n):]
        for t in h:
            if t < 0 or t >= len(x) or t in seen:
                continue
            seen.add(t)
            x[t] = np.float32(x[t] / np.float32(repeat_penalty)) if x[t] > 0 else np.float32(x[t] * np.float32(repeat_penalty))
    return x


def sample(logits, history, temperature, top_k, top_p, repeat_penalty, repeat_last_n, u):
    x = penalize(logits, history, repeat_penalty, repeat_last_n)
    if temperature <= 0:
        return int(np.argmax(x))
    n = len(x)
    k = min(top_k, n) if top_k > 0 else n
    order = np.lexsort((np.arange(n), -x.astype(np.float64)))[:k]  # value descending, index ascending
    vals = x[order]
    mx = vals[0]
    w = np.exp((vals - mx) / np.float32(temperature)).astype(np.float32)
    total_all = float(np.sum(w.astype(np.float64)))
    cum, keep = 0.0, k
    for i in range(k):
        cum += float(w[i]) / total_all
        if cum >= top_p:
            keep = i + 1
            break
    total = 0.0
    for i in range(keep):
        total += float(w[i])
    r = u * total
    for i in range(keep):
        r -= float(w[i])
        if r <= 0:
            return int(order[i])
    return int(order[keep - 1])
