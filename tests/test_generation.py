"""Known-answer tests of the host sampling / MTP acceptance logic, restating
the reference's own tests (packages/engine/test/generation.test.ts and
packages/engine/test/mtp-generation.test.ts) case by case.  Runs on CPU."""
import pytest

from heliopause_b200 import generation as g


def _c(*pairs):
    return [g.Candidate(i, v) for i, v in pairs]


def _dist(*pairs):
    return g.MtpTokenDistribution([(i, float(v)) for i, v in pairs], 16)


def _verification(dists):
    # mtp-generation.test.ts:77-92
    tops = [d.tokens[0][0] for d in dists]
    return g.MtpVerification(tops, dists, dists[-1], tops[-1])


def _seq(*values):
    # mtp-generation.test.ts:94-97: a fixed draw sequence, then 0
    it = iter(values)
    return lambda: next(it, 0.0)


def test_defaults_follow_the_gemma4_config():
    # generation.test.ts:12-30
    r = g.resolve_generation_sampling_options()
    assert g.DEFAULT_GENERATION_CONFIG == {"doSample": True, "temperature": 1.0, "topP": 0.95, "topK": 64,
                                           "bosTokenId": 2, "eosTokenIds": [1, 106, 50], "padTokenId": 0}
    assert (r.do_sample, r.temperature, r.top_p, r.top_k, r.logits_top_k) == (True, 1.0, 0.95, 64, 64)
    assert r.seed == g.DEFAULT_SAMPLING_SEED


def test_validation_and_greedy_top1():
    # generation.test.ts:32-41
    assert g.resolve_generation_sampling_options(do_sample=False, top_k=64).logits_top_k == 1
    assert g.resolve_generation_sampling_options(temperature=0, top_k=64).logits_top_k == 1
    assert g.resolve_generation_sampling_options(top_k=64.9).top_k == 64
    with pytest.raises(ValueError, match="temperature"):
        g.resolve_generation_sampling_options(temperature=-1)
    with pytest.raises(ValueError, match="topP"):
        g.resolve_generation_sampling_options(top_p=0)
    with pytest.raises(ValueError, match="topP"):
        g.resolve_generation_sampling_options(top_p=1.1)
    with pytest.raises(ValueError, match="topK"):
        g.resolve_generation_sampling_options(top_k=0)


def test_rng_first_draw_and_non_greedy_pick():
    # generation.test.ts:43-64
    rng = g.create_deterministic_rng(g.DEFAULT_SAMPLING_SEED)
    assert rng() == 0.9744378970935941
    opt = g.SamplingOptions(True, 1.0, 0.8, 4)
    assert g.sample_next_token(_c((10, 3), (11, 2), (12, 1), (13, 0)), opt,
                               g.create_deterministic_rng(g.DEFAULT_SAMPLING_SEED)) == 11


def test_rng_state_is_the_state_before_the_next_draw():
    # the device sampler draws from rng.state() and the host copy then calls
    # rng() once: a generator restarted from that state makes the same draw,
    # and the stream continues identically
    rng = g.create_deterministic_rng(g.DEFAULT_SAMPLING_SEED)
    for _ in range(5):
        rng()
    s0 = rng.state()
    assert 0 <= s0 < 2 ** 32
    again = g.create_deterministic_rng(s0)
    assert [rng() for _ in range(8)] == [again() for _ in range(8)]
    assert rng.state() == again.state() == (s0 + 8 * 0x6D2B79F5) % 2 ** 32


def test_top_p_keeps_boundary_token_and_greedy_returns_top1():
    # generation.test.ts:66-81
    cands = _c((10, 3), (11, 2), (12, 1))
    assert g.sample_next_token(cands, g.SamplingOptions(False, 1.0, 0.1, 3), lambda: 0.99) == 10
    assert g.sample_next_token(cands, g.SamplingOptions(True, 1.0, 0.8, 3), lambda: 0.99) == 11


MTP_SAMPLING = g.SamplingOptions(True, 1.0, 1.0, 2)  # mtp-generation.test.ts:11-16


def test_mtp_accepts_drafts_and_samples_bonus():
    # mtp-generation.test.ts:18-37
    a = g.accept_mtp_draft(g.MtpProposal([1], [_dist((1, 0), (2, 0))]),
                           _verification([_dist((1, 2), (2, 0)), _dist((3, 0), (4, 0))]), MTP_SAMPLING,
                           _seq(0.1, 0.2))
    assert (a.accepted_draft_length, a.next_token_id, a.committed_length, a.accepted_all_drafts, a.recovered) == \
        (1, 3, 2, True, False)


def test_mtp_rejects_and_samples_recovered():
    # mtp-generation.test.ts:39-58
    a = g.accept_mtp_draft(g.MtpProposal([1], [_dist((1, 4), (2, 0))]),
                           _verification([_dist((1, 0), (2, 4)), _dist((3, 0), (4, 0))]), MTP_SAMPLING,
                           _seq(0.5, 0.1))
    assert (a.accepted_draft_length, a.next_token_id, a.committed_length, a.accepted_all_drafts, a.recovered) == \
        (0, 2, 1, False, True)


def test_mtp_distribution_sampling_uses_constraints():
    # mtp-generation.test.ts:60-68
    assert g.sample_mtp_token_distribution(_dist((10, 10), (11, 9), (12, 8)), g.SamplingOptions(True, 1.0, 1.0, 1),
                                           _seq(0.99)) == 10


def test_greedy_acceptance_paths():
    # mtp-generation.ts:199-228
    a = g.accept_greedy_mtp_draft([5, 6, 7], [5, 6, 9, 4])
    assert (a.accepted_draft_length, a.next_token_id, a.committed_length, a.accepted_all_drafts) == (2, 9, 3, False)
    a = g.accept_greedy_mtp_draft([5, 6], [5, 6, 8])
    assert (a.accepted_draft_length, a.next_token_id, a.committed_length, a.accepted_all_drafts) == (2, 8, 3, True)
    with pytest.raises(ValueError, match="bonus"):
        g.accept_greedy_mtp_draft([5], [5])


def test_target_verification_from_topk_rows():
    v = g.target_verification([[7, 3], [9, 1]], [[2.0, 1.0], [5.0, 0.5]], 16, base_position=100)
    assert v.target_token_ids == [7, 9] and v.bonus_token_id == 9
    assert v.target_distributions[0].tokens == [(7, 2.0), (3, 1.0)]
    assert v.bonus_distribution is v.target_distributions[-1]
