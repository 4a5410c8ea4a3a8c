"""Offline GPTQ quantisation of an HF checkpoint (reference: scripts/quantize_gptq.py).

GPTQ (Frantar et al., 2022, "GPTQ: Accurate Post-Training Quantization for Generative
Pre-trained Transformers") quantises one linear layer at a time so that the layer's output on
calibration inputs changes as little as possible: with H = 2 X^T X over the calibration
activations, columns of W are quantised in order and each column's rounding error is spread
over the not-yet-quantised columns through the upper Cholesky factor of H^-1.

``quantize_checkpoint`` runs the decoder layer by layer: it records the inputs of layer i,
accumulates H for every linear of the layer from those inputs, quantises them, and runs the
quantised layer to produce the inputs of layer i + 1. The output directory is a GPTQ checkpoint
(qweight / qzeros / scales / g_idx per linear, fp16 elsewhere, ``quantization_config`` in
config.json) that ``models/gptq.py`` and HF-style loaders read.

Mixed precision: ``--rule REGEX=METHOD`` (first match on the linear's name wins, else
``--bits``) picks per layer ``gptq4`` / ``gptq8`` (GPTQ at 4 / 8 bits), ``e8`` (E8 lattice vectors, one
byte per 8 weights, models/e8.py, quantised with the same error feedback: each 8-column block takes its
nearest codebook vector and the block's error is spread over the later columns through the
Cholesky factor, the block form of the update) or ``bf16`` (kept). E8 layers are written as
``e8_indices`` / ``e8_scales`` / ``e8_offsets`` with one ``e8_codebook``, 8-bit layers as the
GPTQ tensors at 8 bits, and ``quantization_config`` records ``has_e8``, ``mixed_precision`` and
``modules_not_quantized``.

  python -m b200serve.models.gptq_quantize --model DIR --output DIR [--bits 4] [--group 128]
      [--act-order] [--samples 64] [--seqlen 512] [--device cuda] [--rule 'mlp[.]down=e8' ...]
"""

from __future__ import annotations

import argparse
import json
import os
import re
import shutil

import torch


# ------------------------------------------------------------------ one matrix
def quant_grid(w: torch.Tensor, bits: int):
    """Asymmetric min-max grid per row of ``w`` [N, g]: (scale [N], zero [N] integer).

    The scale is rounded to fp16 (the precision the checkpoint stores), and the zero is at least
    1: the GPTQ v1 format stores zero - 1 in an unsigned field, so a row with no negative weight
    gets the grid [-scale, (maxq - 1) * scale] instead of [0, maxq * scale]."""
    maxq = (1 << bits) - 1
    lo = torch.clamp(w.min(1).values, max=0.0)
    hi = torch.clamp(w.max(1).values, min=0.0)
    flat = (hi - lo) == 0
    lo[flat], hi[flat] = -1.0, 1.0
    nonneg = lo == 0
    scale = torch.where(nonneg, hi / (maxq - 1), (hi - lo) / maxq)
    scale = scale.half().float().clamp_min(1e-8)
    zero = torch.clamp(torch.round(-lo / scale), 1, maxq)
    return scale, zero


def _rtn(w, scale, zero, maxq):
    q = torch.clamp(torch.round(w / scale) + zero, 0, maxq)
    return q, scale * (q - zero)


def gptq_matrix(W: torch.Tensor, H: torch.Tensor, bits: int = 4, group: int = 128, damp: float = 0.01,
                block: int = 128, act_order: bool = False):
    """Quantise W [N, K] (fp32) given H [K, K]. Returns (q int32 [N, K], scales [G, N],
    zeros [G, N] (integer values), g_idx [K] int32), with G = K / group and
    W_hat[n, k] = scales[g_idx[k], n] * (q[n, k] - zeros[g_idx[k], n])."""
    W = W.clone().float()
    H = H.clone().float()
    N, K = W.shape
    maxq = (1 << bits) - 1
    dead = torch.diag(H) == 0
    H[dead, dead] = 1.0
    W[:, dead] = 0.0
    perm = torch.argsort(torch.diag(H), descending=True) if act_order else torch.arange(K, device=W.device)
    W, H = W[:, perm], H[perm][:, perm]
    H += damp * torch.mean(torch.diag(H)) * torch.eye(K, device=W.device)
    U = torch.linalg.cholesky(torch.cholesky_inverse(torch.linalg.cholesky(H)), upper=True)   # chol of H^-1
    Q = torch.zeros(N, K, dtype=torch.int32, device=W.device)
    G = (K + group - 1) // group
    scales = torch.zeros(G, N, device=W.device)
    zeros = torch.zeros(G, N, device=W.device)
    for b0 in range(0, K, block):
        b1 = min(K, b0 + block)
        Wb = W[:, b0:b1].clone()
        Eb = torch.zeros_like(Wb)
        Ub = U[b0:b1, b0:b1]
        for i in range(b1 - b0):
            c = b0 + i
            if c % group == 0:                       # grid of the group starting here (current values)
                gs, gz = quant_grid(torch.cat([Wb[:, i:], W[:, b1:]], 1)[:, :group], bits)
                scales[c // group], zeros[c // group] = gs, gz
            s, z = scales[c // group], zeros[c // group]
            q, wq = _rtn(Wb[:, i], s, z, maxq)
            Q[:, c] = q.to(torch.int32)
            err = (Wb[:, i] - wq) / Ub[i, i]
            Wb[:, i:] -= err[:, None] * Ub[i, i:][None, :]
            Eb[:, i] = err
        W[:, b1:] -= Eb @ U[b0:b1, b1:]
    inv = torch.argsort(perm)
    g_idx = (torch.arange(K, device=W.device) // group)[inv].to(torch.int32)   # group of original column
    return Q[:, inv], scales, zeros, g_idx


def e8_gptq_matrix(W: torch.Tensor, H: torch.Tensor, codebook: torch.Tensor, group: int = 128,
                   damp: float = 0.01):
    """E8 vector quantisation of W [N, K] with GPTQ error feedback over 8-column blocks. Each
    group's (scale, offset) is set from the group's current values when the group starts (offset
    = mean, scale = largest deviation); a block's error E moves the later columns by
    -E U_bb^-1 U_b,later (U the upper Cholesky factor of H^-1). Returns (indices uint8 [N, K/8],
    scales fp16 [N, G], offsets fp16 [N, G])."""
    from b200serve.models import e8 as E8
    W = W.clone().float()
    H = H.clone().float()
    N, K = W.shape
    assert K % group == 0 and group % 8 == 0
    dead = torch.diag(H) == 0
    H[dead, dead] = 1.0
    W[:, dead] = 0.0
    H += damp * torch.mean(torch.diag(H)) * torch.eye(K, device=W.device)
    U = torch.linalg.cholesky(torch.cholesky_inverse(torch.linalg.cholesky(H)), upper=True)
    cb = codebook.float().to(W.device)
    G = K // group
    idx = torch.zeros(N, K // 8, dtype=torch.uint8, device=W.device)
    scales = torch.zeros(N, G, device=W.device)
    offsets = torch.zeros(N, G, device=W.device)
    for c in range(0, K, 8):
        gi = c // group
        if c % group == 0:
            grp = W[:, c:c + group]
            o = grp.mean(1)
            s = (grp - o[:, None]).abs().amax(1).clamp(min=1e-10)
            # the checkpoint stores fp16; quantise against the stored values
            scales[:, gi], offsets[:, gi] = s.half().float(), o.half().float()
        s, o = scales[:, gi], offsets[:, gi]
        blk = W[:, c:c + 8]
        j = E8.nearest((blk - o[:, None]) / s[:, None], cb)
        idx[:, c // 8] = j.to(torch.uint8)
        err = blk - (cb[j] * s[:, None] + o[:, None])
        if c + 8 < K:
            X = torch.linalg.solve_triangular(U[c:c + 8, c:c + 8], err, upper=True, left=False)
            W[:, c + 8:] -= X @ U[c:c + 8, c + 8:]
    return idx, scales.to(torch.float16), offsets.to(torch.float16)


def rtn_matrix(W: torch.Tensor, bits: int = 4, group: int = 128):
    """Round-to-nearest on the same grid (the baseline GPTQ improves on)."""
    N, K = W.shape
    maxq = (1 << bits) - 1
    Q = torch.zeros(N, K, dtype=torch.int32)
    G = (K + group - 1) // group
    scales, zeros = torch.zeros(G, N), torch.zeros(G, N)
    for gi in range(G):
        sl = slice(gi * group, min(K, (gi + 1) * group))
        s, z = quant_grid(W[:, sl].float(), bits)
        scales[gi], zeros[gi] = s, z
        Q[:, sl] = _rtn(W[:, sl].float(), s[:, None], z[:, None], maxq)[0].to(torch.int32)
    return Q, scales, zeros, (torch.arange(K) // group).to(torch.int32)


def dequant(Q, scales, zeros, g_idx) -> torch.Tensor:
    gi = g_idx.long()
    return scales[gi].t() * (Q.float() - zeros[gi].t())


# ------------------------------------------------------------------ checkpoint format
def pack_gptq(Q: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor, g_idx: torch.Tensor, bits: int) -> dict:
    """GPTQ tensors (v1 zero convention: the stored zero is zero - 1) for W [N, K]."""
    N, K = Q.shape
    p = 32 // bits
    assert K % p == 0 and N % p == 0, "K and N must be multiples of 32 / bits"
    qt = Q.t().contiguous().to(torch.int64)                       # [K, N]
    shifts = (torch.arange(p, dtype=torch.int64) * bits).view(1, p, 1)
    qweight = (qt.view(K // p, p, N) << shifts).sum(1)
    z = zeros.to(torch.int64) - 1                                # [G, N]; quant_grid keeps zero >= 1
    assert int(z.min()) >= 0, "GPTQ v1 zeros must be >= 1"
    zshift = (torch.arange(p, dtype=torch.int64) * bits).view(1, 1, p)
    qzeros = (z.view(z.shape[0], N // p, p) << zshift).sum(2)
    def to32(t):                                                 # uint32 bit pattern as int32
        t = t & 0xFFFFFFFF
        return torch.where(t >= (1 << 31), t - (1 << 32), t).to(torch.int32)
    return {"qweight": to32(qweight), "qzeros": to32(qzeros),
            "scales": scales.to(torch.float16), "g_idx": g_idx.to(torch.int32)}


def _plus_one_zeros(qzeros: torch.Tensor, bits: int) -> torch.Tensor:
    """GPTQ v1 zeros (zero - 1 per field) -> the zeros themselves (the ``_q8`` tensors' convention)."""
    p = 32 // bits
    z = qzeros.to(torch.int64) & 0xFFFFFFFF
    f = torch.stack([(z >> (bits * i)) & ((1 << bits) - 1) for i in range(p)], -1) + 1
    assert int(f.max()) < (1 << bits)
    w = (f << (torch.arange(p, dtype=torch.int64) * bits)).sum(-1)
    return torch.where(w >= (1 << 31), w - (1 << 32), w).to(torch.int32)


# ------------------------------------------------------------------ whole checkpoint
class _Stop(Exception):
    pass


def _skip(name: str) -> bool:
    """Linears kept in full precision: the MoE router (tiny and routing-critical)."""
    return name.endswith("mlp.gate") or "router" in name


def calibration_ids(tokenizer, vocab: int, samples: int, seqlen: int, text_file: str = None, seed: int = 0):
    """[samples, seqlen] token ids: windows of a text file when given, else uniform random ids."""
    g = torch.Generator().manual_seed(seed)
    if text_file and tokenizer is not None:
        with open(text_file, encoding="utf-8", errors="replace") as fh:
            ids = tokenizer.encode(fh.read(), add_special_tokens=False)
        if len(ids) > seqlen:
            starts = torch.randint(0, len(ids) - seqlen, (samples,), generator=g).tolist()
            return torch.tensor([ids[s:s + seqlen] for s in starts])
    return torch.randint(0, vocab, (samples, seqlen), generator=g)


METHODS = ("gptq4", "gptq8", "e8", "bf16")


def method_for(name: str, rules, bits: int) -> str:
    """The method of linear ``name``: the first (regex, method) rule that matches, else from bits."""
    for pat, m in rules or ():
        if re.search(pat, name):
            return m
    return {2: "e8", 4: "gptq4", 8: "gptq8", 16: "bf16"}[bits]


@torch.no_grad()
def quantize_checkpoint(model_dir: str, out_dir: str, bits: int = 4, group: int = 128, act_order: bool = False,
                        samples: int = 64, seqlen: int = 512, device: str = None, text_file: str = None,
                        log=print, rules=None, codebook=None) -> dict:
    """GPTQ-quantise every decoder linear of the HF checkpoint at ``model_dir`` into ``out_dir``
    (per-layer methods from ``rules``: [(regex, method)], methods in METHODS; ``codebook`` the
    E8 codebook, default models/e8.lattice_codebook()). Returns {layer linear name: relative
    output error on the calibration inputs}."""
    from b200serve.models import e8 as E8
    for _, m in rules or ():
        assert m in METHODS, f"unknown method {m}"
    cb = (codebook if codebook is not None else E8.lattice_codebook()).float()
    kept, used = [], set()
    from safetensors.torch import save_file
    from transformers import AutoModelForCausalLM
    from b200serve.core.config import TRUST_REMOTE_CODE
    device = torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu"))
    model = AutoModelForCausalLM.from_pretrained(model_dir, dtype=torch.float32,
                                                 trust_remote_code=TRUST_REMOTE_CODE).to(device).eval()
    tok = None
    try:
        from transformers import AutoTokenizer
        tok = AutoTokenizer.from_pretrained(model_dir, trust_remote_code=TRUST_REMOTE_CODE)
    except Exception:
        pass
    ids = calibration_ids(tok, model.config.vocab_size, samples, seqlen, text_file).to(device)
    layers = model.model.layers
    # inputs of layer 0 (hidden states and the layer's keyword arguments), one per sample
    captured = []

    def grab(_mod, args, kwargs):
        captured.append((args[0] if args else kwargs.pop("hidden_states"), dict(kwargs)))
        raise _Stop()
    h = layers[0].register_forward_pre_hook(grab, with_kwargs=True)
    for s in range(ids.shape[0]):
        try:
            model(ids[s:s + 1], use_cache=False)
        except _Stop:
            pass
    h.remove()
    packed, errors = {}, {}
    inputs = captured
    for li, layer in enumerate(layers):
        lins = {n: m for n, m in layer.named_modules() if isinstance(m, torch.nn.Linear) and not _skip(n)}
        hess = {n: torch.zeros(m.in_features, m.in_features, device=device) for n, m in lins.items()}
        seen = {n: 0 for n in lins}
        outs_ref = {}

        def hook(name):
            def f(mod, inp, out):
                x = inp[0].reshape(-1, inp[0].shape[-1]).float()
                n0, n1 = seen[name], x.shape[0]
                hess[name].mul_(n0 / (n0 + n1)).add_(x.t() @ x, alpha=2.0 / (n0 + n1))
                seen[name] = n0 + n1
                outs_ref.setdefault(name, []).append((x, out.reshape(-1, out.shape[-1]).float()))
            return f
        hs = [m.register_forward_hook(hook(n)) for n, m in lins.items()]
        for x, kw in inputs:
            layer(x, **kw)
        for hh in hs:
            hh.remove()
        for n, m in lins.items():
            full = f"model.layers.{li}.{n}"
            meth = method_for(full, rules, bits)
            used.add(meth)
            W = m.weight.data.float()
            if meth == "bf16":
                kept.append(full)
                errors[f"layers.{li}.{n}"] = 0.0
                continue
            if meth == "e8":
                gs = group if W.shape[1] % group == 0 else 32
                idx, sc, of = e8_gptq_matrix(W, hess[n], cb.to(W.device), gs)
                what = E8.dequantize(idx, sc, of, cb.to(W.device), gs).to(m.weight.dtype)
                packed[full] = {"e8_indices": E8.pack_indices(idx.cpu()), "e8_scales": sc.t().contiguous().cpu(),
                                "e8_offsets": of.t().contiguous().cpu()}
            else:
                b = 4 if meth == "gptq4" else 8
                Q, sc, zr, gi = gptq_matrix(W, hess[n], b, group, act_order=act_order)
                what = dequant(Q, sc, zr, gi).to(m.weight.dtype)
                t = pack_gptq(Q.cpu(), sc.cpu(), zr.cpu(), gi.cpu(), b)
                assert not (b == 4 and bits == 8), "4-bit layers need --bits 4 (8-bit layers then use the _q8 names)"
                if b == 8 and bits != 8:                  # 8-bit layers next to 4-bit ones: the _q8 names, zero as is
                    t = {"qweight_q8": t["qweight"], "scales_q8": t["scales"], "g_idx_q8": t["g_idx"],
                         "qzeros_q8": _plus_one_zeros(t["qzeros"], 8)}
                packed[full] = t
            xs = torch.cat([x for x, _ in outs_ref[n]])
            ref = xs @ W.t()
            errors[f"layers.{li}.{n}"] = ((xs @ what.float().t() - ref).norm() / ref.norm()).item()
            m.weight.data.copy_(what)
        nxt = []
        for x, kw in inputs:                         # the quantised layer feeds the next one
            y = layer(x, **kw)
            nxt.append((y[0] if isinstance(y, tuple) else y, kw))
        inputs = nxt
        log(f"gptq: layer {li} done, worst rel. output error {max(v for k, v in errors.items() if f'layers.{li}.' in k):.4f}")
    # write the checkpoint: quantised linears as GPTQ tensors, everything else fp16
    os.makedirs(out_dir, exist_ok=True)
    tensors = {}
    for k, v in model.state_dict().items():
        base = k[:-len(".weight")] if k.endswith(".weight") else None
        if base is not None and base in packed:
            for suffix, t in packed[base].items():
                tensors[f"{base}.{suffix}"] = t.contiguous()
        else:
            tensors[k] = v.detach().to(torch.float16).cpu().contiguous()
    if "e8" in used:
        tensors["e8_codebook"] = cb.cpu().contiguous()
    save_file(tensors, os.path.join(out_dir, "model.safetensors"), metadata={"format": "pt"})
    cfg = model.config.to_dict()
    main_bits = 8 if bits == 8 else 4
    cfg["quantization_config"] = {"quant_method": "gptq", "bits": main_bits, "group_size": group,
                                  "desc_act": act_order, "sym": False, "checkpoint_format": "gptq",
                                  "mixed_precision": len(used) > 1 or bool(kept) or "e8" in used,
                                  "has_e8": "e8" in used,
                                  "has_q8": any(k.endswith("qweight_q8") for t in packed.values() for k in t),
                                  "modules_not_quantized": kept}
    cfg["torch_dtype"] = "float16"
    with open(os.path.join(out_dir, "config.json"), "w") as fh:
        json.dump(cfg, fh, indent=1)
    for f in os.listdir(model_dir):
        if f.startswith("tokenizer") or f in ("special_tokens_map.json", "vocab.json", "merges.txt",
                                              "generation_config.json"):
            shutil.copy(os.path.join(model_dir, f), os.path.join(out_dir, f))
    return errors


def main(argv=None):
    ap = argparse.ArgumentParser("b200serve GPTQ quantiser")
    ap.add_argument("--model", required=True)
    ap.add_argument("--output", required=True)
    ap.add_argument("--bits", type=int, default=4, choices=[2, 4, 8], help="2: E8 vectors, 4 / 8: GPTQ")
    ap.add_argument("--group", type=int, default=128)
    ap.add_argument("--act-order", action="store_true")
    ap.add_argument("--samples", type=int, default=64)
    ap.add_argument("--seqlen", type=int, default=512)
    ap.add_argument("--device", default=None)
    ap.add_argument("--text", default=None, help="calibration text file (default: random token ids)")
    ap.add_argument("--rule", action="append", default=[],
                    help="REGEX=METHOD (gptq4, gptq8, e8, bf16) for the linears whose name matches")
    a = ap.parse_args(argv)
    rules = [tuple(r.rsplit("=", 1)) for r in a.rule]
    errs = quantize_checkpoint(a.model, a.output, a.bits, a.group, a.act_order, a.samples, a.seqlen, a.device, a.text,
                               rules=rules)
    print(json.dumps({"layers": len(errs), "max_rel_output_error": max(errs.values())}))


if __name__ == "__main__":
    main()
