"""Seeded multi-step verification scenarios (region blocks with true texts)."""
import numpy as np

VOCAB = 1000
EOS = VOCAB          # outside the model's wrong-token range [1, VOCAB)
PAD = 0


def _perturb(rng, truth, p_sub, p_del, p_ins):
    out = []
    for t in truth:
        u = rng.random()
        if u < p_del:
            continue
        if u < p_del + p_sub:
            out.append(int(rng.integers(1, VOCAB)))
        else:
            out.append(int(t))
        if rng.random() < p_ins:
            out.append(int(rng.integers(1, VOCAB)))
    return out


def make_loop_case(seed, n_blocks=6):
    """prompts, truths, drafts: good, noisy, useless drafts and one periodic
    text that ends in the repetition stop."""
    rng = np.random.default_rng(seed)
    prompts, truths, drafts = [], [], []
    for b in range(n_blocks):
        prompts.append([int(x) for x in rng.integers(1, VOCAB, int(rng.integers(12, 40)))])
        n = int(rng.integers(30, 140))
        kind = b % 4
        if kind == 3:                                      # periodic text
            unit = [int(x) for x in rng.integers(1, VOCAB, 5)]
            truth = (unit * 40)[:150]
            draft = _perturb(rng, truth[:60], 0.02, 0.0, 0.0)
        else:
            truth = [int(x) for x in rng.integers(1, VOCAB, n)]
            if kind == 0:                                  # good draft
                draft = _perturb(rng, truth, 0.02, 0.01, 0.01)
            elif kind == 1:                                # noisy draft
                draft = _perturb(rng, truth, 0.08, 0.05, 0.05)
            else:                                          # useless draft
                draft = [int(x) for x in rng.integers(1, VOCAB, n // 2)]
        truths.append(np.asarray(truth, dtype=np.int64))
        drafts.append(draft)
    return prompts, truths, drafts


def logits_model(model, seed=0):
    """Dense logits ``[Q, VOCAB + 1]`` around ``model``'s tokens, for the
    logit-ratio rules: the model's token gets 8.0, every other entry a value
    k / 8, k in [-48, 48), drawn from the row's token and position (all
    exact in bf16), so a draft token's ratio is k / 64."""
    def fn(input_ids, position_ids, allowed, kv_tokens):
        nxt = np.asarray(model(input_ids, position_ids, allowed, kv_tokens), dtype=np.int64)
        q = len(nxt)
        out = np.empty((q, VOCAB + 1), dtype=np.float32)
        for r in range(q):
            g = np.random.default_rng((seed, int(input_ids[r]), int(position_ids[r])))
            out[r] = g.integers(-48, 48, VOCAB + 1) / 8.0
        out[np.arange(q), nxt] = 8.0
        return out
    return fn
