"""Greedy identity of self-speculative decoding through the hot path.

A Qwen3-1.7B-shaped model with random-init bf16 weights decodes a batch of
synthetic prompts with the fixed-draft schedule (draft length 4, a 32-page
sparse budget of a 2048-token context, 8 recent pages, refresh layer -2),
every attention, append, page selection and spill through libaspire_b200.
ASPIRE's verification makes its greedy output the target model's greedy
output (aspire/engine/runtime.py:765-783), so:

* two runs from the same prefill state emit identical tokens (sha256), and a
  run with every step eager emits the same tokens as the CUDA-graph run;
* every emitted token is the target's greedy choice given the emitted
  prefix: feeding the output back through full causal attention, the logit
  of each emitted token is the maximum, or within GAP_TOL of it where the two
  computations differ in bf16 rounding (near-ties);
* plain greedy decoding (draft length 0, every step a full-attention step
  through the same ops) passes the same check, and the speculative output is
  compared with it token for token;
* with a budget covering the whole context, the draft rows attend every
  page through their draft tables, so their drafts are the target's own
  greedy tokens and nearly all are accepted: this checks the draft path
  (seeding, re-selection every step, the table ending at the newest page,
  sparse attention through the tables) end to end.  With the 32-page budget
  and random-init weights the drafts are rarely right: the attention output
  of such a model is a small, context-spread part of the residual stream, so
  which 32 of 128 pages a row sees moves the logits by more than the gaps
  between the top bf16 logits.
"""

import numpy as np
import pytest
import torch

from aspire_b200.spec_decode import PRESETS, DenseModel, SpecDecoder, compare_sequences, synthetic_prompts, token_sha256

pytestmark = pytest.mark.gpu

B, P, G = 8, 2048, 48
GAP_TOL = 0.25


@pytest.fixture(scope="module")
def model(cuda_device):
    return DenseModel(PRESETS["qwen3-1.7b"], cuda_device, seed=0)


def _check_greedy(dec, tokens, label):
    agree, gaps = dec.teacher_forced_check(P, tokens)
    print(f"{label}: teacher-forced agreement {agree.mean():.4f}, max gap {gaps.max():.4f}, "
          f"gaps>0: {np.sort(gaps[gaps > 0])[-8:]}")
    assert gaps.max() <= GAP_TOL, (label, float(gaps.max()))
    return agree, gaps


def test_speculative_output_is_target_greedy(model):
    prompts = synthetic_prompts(B, P, model.cfg.vocab, seed=0)
    dec = SpecDecoder(model, batch=B, prompt_len=P, max_new=G, draft_len=4, budget_pages=32, recent_pages=8)
    g0 = dec.prefill(prompts)
    a = dec.generate()
    dec.restart(g0)
    b = dec.generate()
    assert token_sha256(a["tokens"]) == token_sha256(b["tokens"])
    dec.restart(g0)
    dec.use_graphs = False
    c = dec.generate()
    assert np.array_equal(a["tokens"], c["tokens"]), "CUDA-graph replay differs from eager steps"
    print("spec:", {k: v for k, v in a.items() if k != "tokens"})
    _check_greedy(dec, a["tokens"], "speculative")

    ar = SpecDecoder(model, batch=B, prompt_len=P, max_new=G, draft_len=0, budget_pages=32, recent_pages=8)
    g0_ar = ar.prefill(prompts)
    assert np.array_equal(g0, g0_ar)
    r = ar.generate()
    _check_greedy(ar, r["tokens"], "plain greedy")
    cmp = compare_sequences(a["tokens"], r["tokens"])
    print("speculative vs plain greedy:", cmp)


def test_full_budget_drafts_are_accepted(model):
    """Budget = every page of the context: drafting sees the full context
    through the draft tables, so nearly every draft is accepted."""
    prompts = synthetic_prompts(B, P, model.cfg.vocab, seed=1)
    pages = (P + G + 4 + 15) // 16
    dec = SpecDecoder(model, batch=B, prompt_len=P, max_new=G, draft_len=4, budget_pages=pages, recent_pages=8)
    dec.prefill(prompts)
    a = dec.generate()
    rate = a["accepted_drafts"] / max(a["verify_rows"] * 4, 1)
    print("full budget:", {k: v for k, v in a.items() if k != "tokens"}, "acceptance", round(rate, 4))
    assert rate >= 0.8, rate
    _check_greedy(dec, a["tokens"], "full budget")


def test_random_draft_lengths_mix_steps_and_stay_greedy(model):
    """Per-row draft lengths drawn from 2..6 after every verification (config
    3's asynchronous interleaving): the rows drift apart, so most steps hold
    drafting and verifying rows together, and the output is still a greedy
    decode of the same prompts.  It is compared with plain greedy decoding
    token for token: the split-KV chunk of a row depends on the batch around
    it (a mixed step cuts the verify rows into one piece per SM, a plain
    step into 512-token chunks), so the two sum a row's attention in a
    different order, and where the top two bf16 logits are that close the
    argmax can differ.  Rows may therefore part only at such a near-tie:
    at the first divergence both emitted tokens are within GAP_TOL of the
    teacher-forced maximum of their common prefix."""
    prompts = synthetic_prompts(B, P, model.cfg.vocab, seed=2)
    dec = SpecDecoder(model, batch=B, prompt_len=P, max_new=G, draft_len=(2, 6), budget_pages=32, recent_pages=8,
                      draft_seed=3)
    g0 = dec.prefill(prompts)
    a = dec.generate()
    print("random lengths:", {k: v for k, v in a.items() if k != "tokens"})
    assert a["steps"]["mixed"] > a["steps"]["draft"] + a["steps"]["verify"], a["steps"]
    dec.restart(g0)
    b = dec.generate()
    assert np.array_equal(a["tokens"], b["tokens"])
    _, gaps_a = _check_greedy(dec, a["tokens"], "random lengths")
    ar = SpecDecoder(model, batch=B, prompt_len=P, max_new=G, draft_len=0, budget_pages=32, recent_pages=8)
    ar.prefill(prompts)
    r = ar.generate()
    _, gaps_r = _check_greedy(ar, r["tokens"], "plain greedy")
    cmp = compare_sequences(a["tokens"], r["tokens"])
    print("random lengths vs plain greedy:", cmp)
    for row, d in enumerate(cmp["first_divergence"]):
        if d < 0:
            continue
        # gaps[:, j] belongs to token j + 1; the first token comes from the shared prefill
        assert d >= 1, (row, d)
        ga, gr = float(gaps_a[row, d - 1]), float(gaps_r[row, d - 1])
        assert ga <= GAP_TOL and gr <= GAP_TOL, (row, d, ga, gr)
