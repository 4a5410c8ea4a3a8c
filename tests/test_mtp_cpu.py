"""MTP speculative decoding: greedy outputs with the head drafting equal plain one-token
decoding (random head: drafts are mostly rejected); with an oracle head whose draft is exactly
the trunk's next prediction every draft is accepted; checkpoint ``mtp.*`` tensors load."""

import torch

from b200serve.core.config import EngineConfig
from b200serve.engine.b200_engine import B200Engine
from b200serve.engine.sampler import SamplingParams
from b200serve.models import mtp as MTP
from b200serve.models import weights as W
from b200serve.models.config import get_model_config

CFG = get_model_config("tiny-qwen2")


def _run(weights, head, prompts, params, spec):
    eng = B200Engine(EngineConfig(model="tiny-qwen2", device="cpu", dtype="float32", cuda_graphs=False,
                                  max_seq=512, max_batch=4, spec_mtp=spec), weights=weights, model_config=CFG,
                     mtp=head)
    try:
        outs = [r.output for r in eng.generate(prompts, params)]
        return outs, dict(eng.scheduler.stats)
    finally:
        eng.unload()


def _prompts(seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(3, 32000, (n,), generator=g).tolist() for n in (9, 23, 40)]


def test_random_head_keeps_greedy_outputs():
    sp = SamplingParams(temperature=0.0, max_tokens=20, ignore_eos=True)
    w = W.random_weights(CFG, seed=1, dtype=torch.float32)
    plain, _ = _run(w, None, _prompts(), sp, False)
    w = W.random_weights(CFG, seed=1, dtype=torch.float32)
    spec, st = _run(w, MTP.random_mtp(CFG, seed=2, dtype=torch.float32), _prompts(), sp, True)
    assert spec == plain
    assert st["spec_steps"] > 0 and st["spec_drafted"] > 0


def _oracle():
    """Trunk layers that add nothing (o and down zero): the hidden stays the token embedding and
    the next token is argmax lm_head(final_norm(E[t])). The head's layer adds nothing either and
    its input is the normalised next-token embedding, so its draft for the token after t is the
    same function of t: every draft matches the trunk."""
    w = W.random_weights(CFG, seed=3, dtype=torch.float32)
    for lw in w.layers:
        lw.o.zero_()
        lw.down.zero_()
    head = MTP.random_mtp(CFG, seed=4, dtype=torch.float32)
    head.layer.o.zero_()
    head.layer.down.zero_()
    H = CFG.hidden_size
    head.eh_proj.zero_()
    head.eh_proj[:, :H] = torch.eye(H)
    head.head_norm.copy_(w.final_norm)
    return w, head


def test_oracle_head_drafts_are_all_accepted():
    sp = SamplingParams(temperature=0.0, max_tokens=24, ignore_eos=True)
    w, head = _oracle()
    spec, st = _run(w, head, _prompts(5), sp, True)
    w, _ = _oracle()
    plain, _ = _run(w, None, _prompts(5), sp, False)
    assert spec == plain
    assert st["spec_drafted"] > 0 and st["spec_accepted"] >= 0.95 * st["spec_drafted"]
    # every accepted draft saves a forward: fewer verify steps than generated tokens
    assert st["spec_steps"] < sum(len(o) for o in spec)


def test_head_loads_from_checkpoint_tensors():
    head = MTP.random_mtp(CFG, seed=6, dtype=torch.float32)
    lw = head.layer
    H, hd, nq, nkv = CFG.hidden_size, CFG.head_dim, CFG.num_heads, CFG.num_kv_heads
    I = CFG.intermediate_size
    gu = lw.gate_up
    from b200serve.models.weights import deinterleave_gate_up
    g, u = deinterleave_gate_up(gu, I)
    sd = {"mtp.fc.weight": head.eh_proj, "mtp.pre_fc_norm_embedding.weight": head.enorm,
          "mtp.pre_fc_norm_hidden.weight": head.hnorm, "mtp.norm.weight": head.head_norm,
          "mtp.layers.0.input_layernorm.weight": lw.input_norm,
          "mtp.layers.0.post_attention_layernorm.weight": lw.post_norm,
          "mtp.layers.0.self_attn.q_proj.weight": lw.qkv[:nq * hd],
          "mtp.layers.0.self_attn.k_proj.weight": lw.qkv[nq * hd:(nq + nkv) * hd],
          "mtp.layers.0.self_attn.v_proj.weight": lw.qkv[(nq + nkv) * hd:],
          "mtp.layers.0.self_attn.q_proj.bias": lw.qkv_bias[:nq * hd],
          "mtp.layers.0.self_attn.k_proj.bias": lw.qkv_bias[nq * hd:(nq + nkv) * hd],
          "mtp.layers.0.self_attn.v_proj.bias": lw.qkv_bias[(nq + nkv) * hd:],
          "mtp.layers.0.self_attn.o_proj.weight": lw.o,
          "mtp.layers.0.mlp.gate_proj.weight": g, "mtp.layers.0.mlp.up_proj.weight": u,
          "mtp.layers.0.mlp.down_proj.weight": lw.down[:, :I]}
    back = MTP.mtp_from_getter(CFG, sd.get, dtype=torch.float32)
    assert torch.equal(back.eh_proj, head.eh_proj) and torch.equal(back.layer.qkv, lw.qkv)
    assert torch.equal(back.layer.gate_up, lw.gate_up) and torch.equal(back.layer.o, lw.o)
    assert MTP.mtp_from_getter(CFG, {}.get) is None
