"""DRY repetition penalty: a token that would extend a repeat of at least the allowed
length is penalised by multiplier * base^(length - allowed); shorter repeats and tokens
that never followed the current suffix are untouched; greedy sampling honours it."""

import torch

from b200serve.engine.sampler import SamplingParams, dry_penalties, sample


def test_penalty_lengths():
    p = SamplingParams(dry_multiplier=0.8, dry_base=1.75, dry_allowed_length=2)
    hist = [1, 2, 3, 4, 9, 1, 2, 3]
    pen = dry_penalties(hist, p)
    assert abs(pen[4] - 0.8 * 1.75 ** 1) < 1e-9      # [1 2 3] then 4 earlier: length 3
    assert 9 not in pen and 1 not in pen
    assert dry_penalties([5, 6, 5], p) == {}          # repeat of length 1 < allowed 2


def test_window_and_off():
    p = SamplingParams(dry_multiplier=1.0, dry_penalty_last_n=4)
    assert dry_penalties([1, 2, 3, 4, 9, 1, 2, 3], p) == {}    # the earlier occurrence is outside the window
    off = SamplingParams(dry_multiplier=0.0)
    assert not off.dry and off.plain


def test_greedy_sampling_applies_dry():
    logits = torch.zeros(1, 16)
    logits[0, 4] = 1.0
    logits[0, 7] = 0.9
    hist = [[1, 2, 3, 4, 9, 1, 2, 3]]
    plain = SamplingParams(temperature=0.0)
    dry = SamplingParams(temperature=0.0, dry_multiplier=0.8)
    assert sample(logits, [plain], hist).item() == 4
    assert sample(logits, [dry], hist).item() == 7
    assert logits[0, 4] == 1.0                        # caller's logits untouched


def test_from_dict_reads_dry_keys():
    sp = SamplingParams.from_dict({"temperature": 0.7, "dry_multiplier": 0.8, "dry_base": 2.0,
                                   "dry_allowed_length": 3, "dry_penalty_last_n": 128})
    assert (sp.dry_multiplier, sp.dry_base, sp.dry_allowed_length, sp.dry_penalty_last_n) == (0.8, 2.0, 3, 128)
    assert sp.dry and not sp.plain
