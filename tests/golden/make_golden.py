"""Generate golden vectors by running the REFERENCE's own code (CPU, fp32).

Run in a container where the reference checkout exists:

    python tests/golden/make_golden.py /path/to/Sparse-Attention-VGGT

It imports saf3r (with one-line stubs for the config packages addict and
omegaconf, which the hot path never uses), calls the reference functions on
seeded inputs, and writes small .npz fixtures next to this script.  The GPU
box never runs this script; tests only read the committed .npz files.

Fixtures:
  block_mean.npz      saf3r/patch/adaptive_block_value.py:16-23 block_mean
  token_layout.npz    saf3r/patch/value_evolving_attention.py:17-20 token_layout
  relevance.npz       saf3r/patch/coarse_sensing.py:25-31 relevance_logits
  select_topk.npz     saf3r/patch/adaptive_block_value.py:42-56 select_block_mask
                      (fast path a == count, no history)
  concentration.npz   saf3r/patch/region_history_attention.py:39-42 concentration
  mask_assembly.npz   saf3r/patch/adaptive_block_value.py:42-91 select_block_mask
                      with value order, history and every attention/count mix,
                      plus the same-pass history update of :389-396
                      (evidence.topk(keep) gathered from the ids); tie-free
                      inputs (continuous scores, distinct history entries)
  attention_*.npz     the known-answer case of
                      tests/test_adaptive_block_value.py:154-184 (inputs rounded
                      to bf16 so the GPU sees the same values), expected output
                      and evidence from that test's fp32 formula
  layer_cpu.npz       AdaptiveBlockValueAttention.forward on CPU
                      (saf3r/patch/adaptive_block_value.py:285-441), i.e. the
                      reference's own CPU kernel branch :371-385, with fixed
                      per-head decisions; captures q/k/v, masks and the
                      pre-projection attention output
"""
import math
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(path):
    for name in ("addict", "omegaconf"):
        if name not in sys.modules:
            sys.modules[name] = types.ModuleType(name)
    sys.modules["addict"].Dict = dict

    class _OmegaConf:
        @staticmethod
        def register_new_resolver(*a, **k):
            pass

    sys.modules["omegaconf"].OmegaConf = _OmegaConf
    sys.modules["omegaconf"].DictConfig = dict
    sys.modules["omegaconf"].ListConfig = list
    sys.path.insert(0, path)
    import saf3r.patch.adaptive_block_value as abv
    from saf3r.patch.coarse_sensing import relevance_logits
    from saf3r.patch.region_history_attention import concentration
    from saf3r.patch.value_evolving_attention import token_layout
    from saf3r.models.official_vggt.layers.attention import Attention
    return abv, relevance_logits, concentration, token_layout, Attention


def bf16_round(x):
    return x.to(torch.bfloat16).float()


def main(ref_path):
    abv, relevance_logits, concentration, token_layout, Attention = _import_reference(ref_path)
    torch.manual_seed(1234)

    # -- block_mean -----------------------------------------------------------
    x = bf16_round(torch.randn(3, 137, 64))
    out = {"x": x.numpy()}
    for block in (32, 64, 128):
        m, pop = abv.block_mean(x, block)
        out["mean_%d" % block] = m.numpy()
        out["pop_%d" % block] = pop.numpy()
    np.savez_compressed(os.path.join(HERE, "block_mean.npz"), **out)

    # -- token_layout -----------------------------------------------------------
    out = {}
    for frames, ppf in ((3, 10), (4, 1369)):
        p, s = token_layout(frames, ppf, 5, "cpu")
        out["patch_%d_%d" % (frames, ppf)] = p.numpy()
        out["special_%d_%d" % (frames, ppf)] = s.numpy()
    np.savez_compressed(os.path.join(HERE, "token_layout.npz"), **out)

    # -- relevance_logits (pooled scores) --------------------------------------
    q = bf16_round(torch.randn(2, 9, 64))
    pk = torch.randn(2, 12, 64)
    np.savez_compressed(os.path.join(HERE, "relevance.npz"), q=q.numpy(), pooled=pk.numpy(),
                        scale=np.float32(0.125),
                        logits=relevance_logits(q, pk, 0.125).numpy())

    # -- top-k selection (fast path of select_block_mask) -----------------------
    scores = torch.rand(6, 11, 40)           # tie-free
    tied = torch.randint(0, 6, (6, 11, 40)).float() / 4   # many ties
    order = torch.arange(40)
    out = {"scores": scores.numpy(), "tied": tied.numpy()}
    for k in (1, 5, 13, 40):
        out["ids_%d" % k] = np.stack(
            [abv.select_block_mask(scores[h], order, k, k)[0].numpy() for h in range(6)])
        out["tied_ids_%d" % k] = np.stack(
            [abv.select_block_mask(tied[h], order, k, k)[0].numpy() for h in range(6)])
    np.savez_compressed(os.path.join(HERE, "select_topk.npz"), **out)

    # -- concentration (mass threshold) ----------------------------------------
    logits = torch.randn(64, 300) * 3.0
    probs = logits.softmax(-1)
    out = {"logits": logits.numpy(), "probs": probs.numpy(),
           "known_probs": np.array([[.25] * 4, [.9, .04, .03, .03]], dtype=np.float32),
           "known_conc": concentration(torch.tensor([[.25] * 4, [.9, .04, .03, .03]])).numpy()}
    for tau in (0.5, 0.8, 0.85, 0.9):
        c = concentration(probs, tau)
        out["conc_%g" % tau] = c.numpy()
        # m recovered from c = 1 - m / nb
        out["m_%g" % tau] = np.rint((1.0 - c.double().numpy()) * probs.shape[1]).astype(np.int64)
    np.savez_compressed(os.path.join(HERE, "concentration.npz"), **out)

    # -- attention known-answer cases -----------------------------------------
    for (d, bq, bk) in ((64, 64, 64), (32, 32, 128), (64, 32, 32), (32, 64, 64)):
        torch.manual_seed(8)
        n = 137
        q = bf16_round(torch.randn(3, n, d))
        npatch = 2 * bk + 43 if bk >= 64 else 2 * bk + 19
        kp = bf16_round(torch.randn(3, npatch, d))
        vp = bf16_round(torch.randn_like(kp))
        ks = bf16_round(torch.randn(3, 7, d))
        vs = bf16_round(torch.randn_like(ks))
        heads = [0, 2]
        counts = [2, 3]
        nq = math.ceil(n / bq)
        patterns = [[0, 2, -1], [1, 2, -1], [0, 1, -1]]
        masks = torch.tensor([[patterns[i % 3] for i in range(nq)], [[0, 1, 2]] * nq],
                             dtype=torch.int32)
        scale = 0.2
        out_ref = torch.full((3, n, d), float("nan"))
        ev_ref = torch.full(masks.shape, -float("inf"))
        for slot, head in enumerate(heads):
            for block in range(nq):
                qr = slice(block * bq, min((block + 1) * bq, n))
                ids = masks[slot, block, :counts[slot]].long()
                ix = (ids[:, None] * bk + torch.arange(bk)).flatten()
                ix = ix[ix < npatch]
                keys = torch.cat((kp[head, ix], ks[head]))
                values = torch.cat((vp[head, ix], vs[head]))
                lg = q[head, qr].float() @ keys.float().T * scale
                out_ref[head, qr] = lg.softmax(-1) @ values.float()
                for j, bid in enumerate(ids):
                    span = (ix // bk == bid)
                    ev_ref[slot, block, j] = lg[:, :len(ix)][:, span].logsumexp(-1).mean()
        np.savez_compressed(
            os.path.join(HERE, "attention_d%d_bq%d_bk%d.npz" % (d, bq, bk)),
            q=q.numpy(), kp=kp.numpy(), vp=vp.numpy(), ks=ks.numpy(), vs=vs.numpy(),
            heads=np.array(heads, np.int32), counts=np.array(counts, np.int32),
            masks=masks.numpy(), scale=np.float32(scale), out=out_ref.numpy(),
            evidence=ev_ref.numpy())

    # -- reference CPU layer path ----------------------------------------------
    torch.manual_seed(21)
    frames, ph, pw, heads, dim = 2, 9, 9, 2, 32
    n = frames * (5 + ph * pw)
    state = abv.AdaptiveBlockState(retention=.5, audit_guard=False, query_block=32, key_block=32,
                                   audit_queries=4)
    state.reset(frames, ph, pw)
    original = Attention(dim=heads * dim, num_heads=heads).eval()
    nb = math.ceil(frames * ph * pw / 32)
    blocks = 3

    def fixed(*args):
        return [dict(rho=.5, blocks=blocks, a_blocks=blocks, alpha=1., use_history=False,
                     audit_nmse=0., audit_p90=0., dense_fallback=False, audit_passed=True)
                for _ in range(heads)]

    captured = {}
    orig_select = abv.select_block_mask

    def recording_select(scores, order, count, a, history=None):
        ids, origin = orig_select(scores, order, count, a, history)
        captured.setdefault("masks", []).append(ids.clone())
        captured.setdefault("routing", []).append(scores.clone())
        return ids, origin

    def qkv_hook(mod, inp, outp):
        captured["qkv"] = outp.detach().clone()

    def proj_hook(mod, inp):
        captured["pre_proj"] = inp[0].detach().clone()

    abv.audited_decisions = fixed
    abv.select_block_mask = recording_select
    h1 = original.qkv.register_forward_hook(qkv_hook)
    h2 = original.proj.register_forward_pre_hook(proj_hook)
    x = torch.randn(1, n, heads * dim)
    with torch.inference_mode():
        abv.AdaptiveBlockValueAttention(original, state, 1).eval()(x)
    h1.remove()
    h2.remove()
    abv.select_block_mask = orig_select
    qkv = captured["qkv"].reshape(1, n, 3, heads, dim).permute(2, 0, 3, 1, 4)[:, 0]
    patches, specials = token_layout(frames, ph * pw, 5, "cpu")
    out_attn = captured["pre_proj"].reshape(n, heads, dim).transpose(0, 1)
    np.savez_compressed(
        os.path.join(HERE, "layer_cpu.npz"),
        q=qkv[0].numpy(), k=qkv[1].numpy(), v=qkv[2].numpy(), patches=patches.numpy(),
        specials=specials.numpy(), masks=torch.stack(captured["masks"]).int().numpy(),
        routing=torch.stack(captured["routing"]).numpy(), out=out_attn.numpy(),
        scale=np.float32(original.scale), block=np.int32(32), nb=np.int32(nb))
    print("golden fixtures written to", HERE)


def mask_assembly(abv):
    """Fixtures of the full select_block_mask and the history update."""
    g = torch.Generator().manual_seed(99)
    rows, blocks, hlen = 24, 150, 20
    scores = torch.randn(rows, blocks, generator=g) * 2.0
    value_order = torch.randperm(blocks, generator=g)
    history = torch.stack([torch.randperm(blocks, generator=g)[:hlen] for _ in range(rows)])
    history[torch.rand(rows, hlen, generator=g) < 0.2] = -1
    cases = [(30, 0, False), (30, 30, False), (30, 12, False), (30, 12, True), (30, 30, True),
             (40, 7, True), (150, 20, True), (30, 1, True)]
    out = {"scores": scores.numpy(), "value_order": value_order.numpy(),
           "history": history.numpy(), "cases": np.asarray(cases, dtype=np.int64)}
    for i, (count, a, use_h) in enumerate(cases):
        ids, origin = abv.select_block_mask(scores, value_order, count, a,
                                            history if use_h else None)
        out["ids_%d" % i] = ids.numpy()
        out["origin_%d" % i] = origin.numpy()
    # same-pass history update on case 3 (adaptive_block_value.py:389-396)
    count, keep = cases[3][0], 10
    evidence = torch.randn(rows, count, generator=g)
    winners = evidence.topk(keep, -1).indices
    out["evidence"] = evidence.numpy()
    out["keep"] = np.int64(keep)
    out["new_history"] = torch.as_tensor(out["ids_3"]).gather(1, winners).numpy()
    np.savez_compressed(os.path.join(HERE, "mask_assembly.npz"), **out)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <path to the reference checkout>")
    main(sys.argv[1])
    mask_assembly(_import_reference(sys.argv[1])[0])
