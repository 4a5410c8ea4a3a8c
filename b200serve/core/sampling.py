"""Sampler preset contract (reference: core/sampling.py:23-111).

Every dict returned is fully explicit: all sampler knobs are present, so the
engine never falls back to an implicit default. The preset table and key
names are the reference's public contract (llama-server parameter names),
so they are reproduced value for value.
"""

SAMPLING_PAYLOAD_KEYS = (
    "temperature",
    "top_k", "top_p", "min_p", "typical_p", "top_n_sigma",
    "repeat_penalty", "repeat_last_n",
    "presence_penalty", "frequency_penalty",
    "dry_multiplier", "dry_base", "dry_allowed_length", "dry_penalty_last_n",
    "xtc_probability", "xtc_threshold",
    "seed", "stop",
)

# Identity settings for every knob; presets are layered on top.
_NEUTRAL = {
    "top_k": 0,
    "top_p": 1.0,
    "min_p": 0.0,
    "typical_p": 1.0,
    "repeat_penalty": 1.0,
    "repeat_last_n": 64,
    "presence_penalty": 0.0,
    "frequency_penalty": 0.0,
    "dry_multiplier": 0.0,
    "dry_base": 1.75,
    "dry_allowed_length": 2,
    "dry_penalty_last_n": -1,
    "xtc_probability": 0.0,
    "xtc_threshold": 0.1,
}

PRESETS = {
    "balanced": {"temperature": 0.7, "top_k": 40, "top_p": 0.9,
                 "min_p": 0.0, "repeat_penalty": 1.0, "dry_multiplier": 0.0},
    "deterministic": {"temperature": 0.0, "top_k": 0, "top_p": 1.0,
                      "min_p": 0.0, "repeat_penalty": 1.0, "dry_multiplier": 0.0},
    "creative": {"temperature": 0.9, "top_k": 50, "top_p": 0.95,
                 "min_p": 0.05, "repeat_penalty": 1.0, "dry_multiplier": 0.8},
    "reference": {"temperature": 1.0, "top_k": 50, "top_p": 1.0,
                  "min_p": 0.0, "repeat_penalty": 1.0, "dry_multiplier": 0.0},
    "agent": {"temperature": 0.6, "top_k": 20, "top_p": 0.95,
              "min_p": 0.0, "repeat_penalty": 1.0, "dry_multiplier": 0.0},
}

# Used when a caller passes sampling=None: balanced minus temperature (the
# caller keeps passing temperature positionally).
DEFAULT_SAMPLING = {k: v for k, v in {**_NEUTRAL, **PRESETS["balanced"]}.items()
                    if k != "temperature"}


def get_preset(name: str, **overrides) -> dict:
    """Fully explicit sampler dict for ``name``; unknown names mean "balanced"."""
    out = dict(_NEUTRAL)
    out.update(PRESETS.get(name) or PRESETS["balanced"])
    out.update(overrides)
    return out


def list_presets() -> tuple:
    """Preset names in display order."""
    return ("balanced", "deterministic", "creative", "reference", "agent")


def filter_payload(sampling: dict) -> dict:
    """Keep only recognised sampler keys (typo hygiene)."""
    return {k: v for k, v in (sampling or {}).items() if k in SAMPLING_PAYLOAD_KEYS}
