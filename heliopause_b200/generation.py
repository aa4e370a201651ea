"""Host-side sampling and MTP draft acceptance around the GPU verify step.

Restates, with the same names (snake_case) and semantics, the host logic of
packages/engine/src/generation.ts and packages/engine/src/mtp-generation.ts:
the deterministic RNG, top-k / top-p / temperature sampling over a top-k
candidate list, and speculative-decoding acceptance of an MTP draft against
the target model's batched verify output.  JavaScript numbers are IEEE f64,
as Python floats are; the RNG's 32-bit integer steps are done modulo 2^32.

The target distributions come from `hpc_model_forward` over
[pending, d1 .. dn] (one batched forward, per-position top-k): see
`target_verification`.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Callable, Sequence

# generation.ts:27-37
DEFAULT_GENERATION_CONFIG = {
    "doSample": True,
    "temperature": 1.0,
    "topP": 0.95,
    "topK": 64,
    "bosTokenId": 2,
    "eosTokenIds": [1, 106, 50],
    "padTokenId": 0,
}
DEFAULT_SAMPLING_SEED = 0x48454C49

_M32 = 0xFFFFFFFF


@dataclass(frozen=True)
class SamplingOptions:
    """ResolvedGenerationSamplingOptions (generation.ts:18-25)."""
    do_sample: bool
    temperature: float
    top_p: float
    top_k: int
    seed: int = DEFAULT_SAMPLING_SEED
    logits_top_k: int = 0


@dataclass(frozen=True)
class Candidate:
    """TopTokenCandidate / TokenProbability (generation.ts:9-16)."""
    id: int
    value: float
    probability: float = 0.0


def resolve_generation_sampling_options(do_sample=None, temperature=None, top_p=None, top_k=None,
                                        seed=None) -> SamplingOptions:
    """generation.ts:39-72, same validation messages."""
    d = DEFAULT_GENERATION_CONFIG
    do_sample = d["doSample"] if do_sample is None else do_sample
    temperature = d["temperature"] if temperature is None else temperature
    top_p = d["topP"] if top_p is None else top_p
    top_k = d["topK"] if top_k is None else top_k
    seed = DEFAULT_SAMPLING_SEED if seed is None else seed
    if not math.isfinite(temperature) or temperature < 0:
        raise ValueError("temperature must be a finite number greater than or equal to 0.")
    if not math.isfinite(top_p) or top_p <= 0 or top_p > 1:
        raise ValueError("topP must be a finite number in the range (0, 1].")
    if not math.isfinite(top_k) or top_k < 1:
        raise ValueError("topK must be a positive finite number.")
    if not math.isfinite(seed):
        raise ValueError("seed must be a finite number.")
    k = max(1, math.floor(top_k))
    greedy = do_sample is False or temperature == 0
    return SamplingOptions(do_sample, temperature, top_p, k, math.floor(seed) & _M32, 1 if greedy else k)


def _imul(a: int, b: int) -> int:
    return (a * b) & _M32


def create_deterministic_rng(seed: float) -> Callable[[], float]:
    """generation.ts:74-83 (a mulberry32-style generator): uniform in [0, 1)."""
    state = math.floor(seed) & _M32

    def rng() -> float:
        nonlocal state
        state = (state + 0x6D2B79F5) & _M32
        v = state
        v = _imul(v ^ (v >> 15), v | 1)
        v ^= (v + _imul(v ^ (v >> 7), v | 61)) & _M32
        return ((v ^ (v >> 14)) & _M32) / 4294967296.0

    # the generator's state before the next draw, for a draw made elsewhere
    # (the device sampler) from the same stream; the caller then calls rng()
    # once to advance this copy past it
    rng.state = lambda: state
    return rng


def _greedy(opt) -> bool:
    return opt.do_sample is False or opt.temperature == 0


def _softmax(values: Sequence[float]) -> list[float]:
    """generation.ts:157-165."""
    mx = -math.inf
    for v in values:
        mx = max(mx, v)
    ex = [math.exp(v - mx) for v in values]
    s = 0.0
    for e in ex:
        s += e
    if s <= 0 or not math.isfinite(s):
        return [1.0 if i == 0 else 0.0 for i in range(len(values))]
    return [e / s for e in ex]


def _apply_top_p(cands: Sequence[Candidate], top_p: float) -> Sequence[Candidate]:
    """generation.ts:135-155: keep the prefix whose probability mass first
    reaches top_p (the boundary token included)."""
    if top_p >= 1 or len(cands) <= 1:
        return cands
    probs = _softmax([c.value for c in cands])
    kept, cum = [], 0.0
    for c, p in zip(cands, probs):
        kept.append(c)
        cum += p
        if cum >= top_p:
            break
    return kept if kept else list(cands[:1])


def token_sampling_distribution(candidates: Sequence[Candidate], opt) -> list[Candidate]:
    """generation.ts:107-133: sort (value desc, id asc), top-k, top-p, then a
    softmax of value / temperature over the survivors."""
    if not candidates:
        raise ValueError("Cannot sample from an empty candidate list.")
    srt = sorted(candidates, key=lambda c: (-c.value, c.id))
    if _greedy(opt):
        t = srt[0]
        return [Candidate(t.id, t.value, 1.0)]
    top = srt[:max(1, math.floor(opt.top_k))]
    nucleus = _apply_top_p(top, opt.top_p)
    probs = _softmax([c.value / opt.temperature for c in nucleus])
    return [Candidate(c.id, c.value, p) for c, p in zip(nucleus, probs)]


def sample_next_token(candidates: Sequence[Candidate], opt, rng: Callable[[], float]) -> int:
    """generation.ts:85-105: inverse-CDF draw over the sampling distribution."""
    dist = token_sampling_distribution(candidates, opt)
    if _greedy(opt):
        return dist[0].id if dist else 0
    draw = rng()
    cum = 0.0
    for c in dist:
        cum += c.probability
        if draw < cum:
            return c.id
    return dist[-1].id


# ------------------------------------------------------------------ MTP ----

@dataclass
class MtpTokenDistribution:
    """MtpTokenDistribution (mtp-target.ts): top-k (id, logit) of one position."""
    tokens: list[tuple[int, float]]
    vocabulary_size: int = 0
    masked: bool = False


@dataclass
class MtpVerification:
    """MtpTargetVerificationResult: per-position target distributions for the
    drafts plus the bonus position."""
    target_token_ids: list[int]
    target_distributions: list[MtpTokenDistribution]
    bonus_distribution: MtpTokenDistribution
    bonus_token_id: int = 0
    base_position: int = 0


@dataclass
class MtpAcceptance:
    """GreedyMtpAcceptance / MtpAcceptance (mtp-generation.ts:34-43)."""
    accepted_draft_length: int
    next_token_id: int
    committed_length: int
    accepted_all_drafts: bool
    recovered: bool = False


@dataclass
class MtpProposal:
    draft_token_ids: list[int]
    draft_distributions: list[MtpTokenDistribution] = field(default_factory=list)


def _mtp_candidates(d: MtpTokenDistribution) -> list[Candidate]:
    return [Candidate(int(i), float(v)) for i, v in d.tokens]


def sample_mtp_token_distribution(d: MtpTokenDistribution, opt, rng) -> int:
    """mtp-generation.ts:139-145."""
    return sample_next_token(_mtp_candidates(d), opt, rng)


def _token_probability(d: MtpTokenDistribution, token_id: int, opt) -> float:
    """mtp-generation.ts:236-242."""
    for c in token_sampling_distribution(_mtp_candidates(d), opt):
        if c.id == token_id:
            return c.probability
    return 0.0


def sample_recovered_token(target: MtpTokenDistribution, draft: MtpTokenDistribution, opt, rng) -> int:
    """mtp-generation.ts:244-273: draw from max(0, p_target - p_draft),
    renormalized; falls back to the target distribution when that is empty."""
    pd = {c.id: c.probability for c in token_sampling_distribution(_mtp_candidates(draft), opt)}
    rec = [(c.id, max(0.0, c.probability - pd.get(c.id, 0.0)))
           for c in token_sampling_distribution(_mtp_candidates(target), opt)]
    rec = [(i, p) for i, p in rec if p > 0]
    total = 0.0
    for _, p in rec:
        total += p
    if total <= 0 or not math.isfinite(total):
        return sample_mtp_token_distribution(target, opt, rng)
    draw = rng() * total
    cum = 0.0
    for i, p in rec:
        cum += p
        if draw < cum:
            return i
    return rec[-1][0]


def accept_greedy_mtp_draft(draft_token_ids: Sequence[int], target_token_ids: Sequence[int]) -> MtpAcceptance:
    """mtp-generation.ts:199-228."""
    for i, d in enumerate(draft_token_ids):
        if i >= len(target_token_ids):
            raise ValueError(f"Missing MTP greedy verification token at draft index {i}.")
        if d != target_token_ids[i]:
            return MtpAcceptance(i, int(target_token_ids[i]), 1 + i, False)
    n = len(draft_token_ids)
    if n >= len(target_token_ids):
        raise ValueError("Missing MTP greedy bonus token.")
    return MtpAcceptance(n, int(target_token_ids[n]), 1 + n, True)


def accept_mtp_draft(proposal: MtpProposal, verification: MtpVerification, opt, rng) -> MtpAcceptance:
    """mtp-generation.ts:147-188: accept draft i while min(1, p_t/p_d) >= u;
    on the first rejection sample the recovered token, else the bonus token."""
    if _greedy(opt):
        a = accept_greedy_mtp_draft(proposal.draft_token_ids, verification.target_token_ids)
        a.recovered = False
        return a
    for i, tok in enumerate(proposal.draft_token_ids):
        if i >= len(proposal.draft_distributions) or i >= len(verification.target_distributions):
            raise ValueError(f"Missing MTP sampling verification data at draft index {i}.")
        dd, td = proposal.draft_distributions[i], verification.target_distributions[i]
        p_d = _token_probability(dd, tok, opt)
        p_t = _token_probability(td, tok, opt)
        if p_d > 0 and min(1.0, p_t / p_d) >= rng():
            continue
        return MtpAcceptance(i, sample_recovered_token(td, dd, opt, rng), 1 + i, False, True)
    n = len(proposal.draft_token_ids)
    return MtpAcceptance(n, sample_mtp_token_distribution(verification.bonus_distribution, opt, rng), 1 + n, True,
                         False)


def target_verification(ids, vals, vocabulary_size: int, base_position: int = 0) -> MtpVerification:
    """Per-position top-k from one batched verify forward ([n+1][k] ids and
    logits, value desc / id asc) as the verify runner's result: position i
    verifies draft i, the last position gives the bonus distribution
    (webgpu/mtp-target-runner.ts:80-161)."""
    ids = [[int(x) for x in row] for row in ids]
    vals = [[float(x) for x in row] for row in vals]
    dists = [MtpTokenDistribution(list(zip(r_i, r_v)), vocabulary_size) for r_i, r_v in zip(ids, vals)]
    tops = [r[0] for r in ids]
    return MtpVerification(tops, dists, dists[-1], tops[-1], base_position)
