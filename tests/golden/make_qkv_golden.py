"""Golden vectors for the fused QKV projection + pooling (vggt_qkv_project_pool).

Run in a container where the reference checkout exists:

    python tests/golden/make_qkv_golden.py /path/to/Sparse-Attention-VGGT

Builds the reference's own attention module (saf3r/models/official_vggt/
layers/attention.py Attention, qk_norm=True, with its RotaryPositionEmbedding2D
of rope.py at frequency 100, as the VGGT aggregator configures it), seeds its
weights, and runs the steps of saf3r/patch/adaptive_block_value.py:297-305 on
CPU with the casts of CUDA bf16 autocast (the reference's inference
precision on a GPU: Linear in bf16, LayerNorm and RoPE in fp32): qkv Linear,
reshape to heads, q_norm / k_norm, RoPE with the aggregator's positions
(specials at (0, 0), patch (y, x) at (y + 1, x + 1)), cast to bf16; then the
token layout split (value_evolving_attention.py token_layout) and the block
means of q and of the patch keys (adaptive_block_value.py block_mean).

Writes qkv.npz: x, w, b (bf16 bit patterns as int16), q_norm / k_norm weight
and bias, pos, q [H, N, 64], k_patch, v_patch, k_special, v_special (bf16
bit patterns), pooled_q [H, QB, 64], pooled_k [H, NB, 64] (fp32).
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)


def main(ref_path):
    from make_golden import _import_reference
    abv, _, _, token_layout, Attention = _import_reference(ref_path)
    from saf3r.models.official_vggt.layers.rope import RotaryPositionEmbedding2D
    torch.manual_seed(4321)
    heads, dim = 4, 256
    frames, gh, gw, spf = 8, 6, 6, 5
    tpf = spf + gh * gw
    n = frames * tpf
    attn = Attention(dim, num_heads=heads, qkv_bias=True, qk_norm=True,
                     rope=RotaryPositionEmbedding2D(frequency=100.0))
    with torch.no_grad():
        attn.qkv.weight.normal_(0, 0.05)
        attn.qkv.bias.normal_(0, 0.1)
        for ln in (attn.q_norm, attn.k_norm):
            ln.weight.normal_(1.0, 0.1)
            ln.bias.normal_(0.0, 0.1)
        # the bf16 parameters the kernel sees (autocast's casts)
        attn.qkv.weight.copy_(attn.qkv.weight.to(torch.bfloat16).float())
        attn.qkv.bias.copy_(attn.qkv.bias.to(torch.bfloat16).float())
    x = torch.randn(1, n, dim).to(torch.bfloat16)
    yy, xx = torch.meshgrid(torch.arange(gh), torch.arange(gw), indexing="ij")
    grid = torch.stack((yy.flatten() + 1, xx.flatten() + 1), -1)
    pos = torch.cat((torch.zeros(spf, 2, dtype=torch.long), grid)).repeat(frames, 1)[None]
    with torch.no_grad():
        # the casts CUDA autocast applies on the GPU (CPU autocast's policy
        # differs: it keeps layer_norm in bf16): the Linear in bf16 (fp32
        # accumulate, bf16 output), layer_norm on fp32 input with fp32 output,
        # so RoPE runs in fp32
        w16, b16 = attn.qkv.weight.to(torch.bfloat16), attn.qkv.bias.to(torch.bfloat16)
        qkv = torch.nn.functional.linear(x, w16, b16)
        qkv = qkv.reshape(1, n, 3, heads, dim // heads).permute(2, 0, 3, 1, 4)
        q, k, v = qkv.unbind(0)
        q, k = attn.q_norm(q.float()), attn.k_norm(k.float())
        q, k = attn.rope(q, pos), attn.rope(k, pos)
    q, k, v = (t[0].to(torch.bfloat16).float() for t in (q, k, v))
    patches, specials = token_layout(frames, gh * gw, spf, torch.device("cpu"))
    kp, vp = k[:, patches], v[:, patches]
    ks, vs = k[:, specials], v[:, specials]
    pooled_q, _ = abv.block_mean(q, 64)
    pooled_k, _ = abv.block_mean(kp, 64)
    bits = lambda t: t.to(torch.bfloat16).view(torch.int16).numpy()  # exact bf16 patterns
    np.savez_compressed(
        os.path.join(HERE, "qkv.npz"),
        x=bits(x[0]), w=bits(attn.qkv.weight.detach()), b=bits(attn.qkv.bias.detach()),
        qn_w=attn.q_norm.weight.detach().numpy(), qn_b=attn.q_norm.bias.detach().numpy(),
        kn_w=attn.k_norm.weight.detach().numpy(), kn_b=attn.k_norm.bias.detach().numpy(),
        ln_eps=np.float32(attn.q_norm.eps), pos=pos[0].numpy().astype(np.int32),
        tokens_per_frame=np.int32(tpf), special_per_frame=np.int32(spf),
        q=bits(q), k_patch=bits(kp), v_patch=bits(vp), k_special=bits(ks), v_special=bits(vs),
        pooled_q=pooled_q.numpy(), pooled_k=pooled_k.numpy())
    print("qkv.npz:", heads, "heads,", n, "tokens; q dtype after autocast steps ok")


if __name__ == "__main__":
    main(sys.argv[1])
