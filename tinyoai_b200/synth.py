"""Seeded synthetic StableLM checkpoints for the benchmark configurations.

Every 2-D weight is drawn N(0, std) (std 0.02, the Hugging Face initializer
range) from its own generator seeded by (seed, tensor index), then encoded
in the requested GGUF format; LayerNorm weights are 1 and biases 0. The same
bytes feed the CUDA backend and the CPU oracle, so both consume identical
inputs. Token ids are drawn uniformly from [3, vocab) with numpy's
default_rng(seed).

Q8_0 encoding follows the GGUF layout the reference decodes (matmul.go:24-34:
a binary16 scale d = max|x|/127 followed by 32 int8 round(x/d)).
"""
import numpy as np

from .checkpoint import stablelm_layer_names

CLIO_3B = dict(model_type="stablelm", vocab_size=65536, hidden_size=2560, intermediate_size=6912,
               num_hidden_layers=32, num_attention_heads=32, num_key_value_heads=32,
               max_position_embeddings=8192, layer_norm_eps=1e-5, rope_theta=10000.0,
               partial_rotary_factor=0.25, use_parallel_residual=True, use_qkv_bias=False,
               qk_layernorm=False, tie_word_embeddings=False, hidden_act="silu",
               bos_token_id=0, eos_token_id=0)


def shapes(c):
    d, h, L = c["hidden_size"], c["intermediate_size"], c["num_hidden_layers"]
    kv = d // c["num_attention_heads"] * c["num_key_value_heads"]
    out = {}
    for l in range(L):
        p = f"model.layers.{l}."
        out[p + "input_layernorm.weight"] = (d,)
        out[p + "input_layernorm.bias"] = (d,)
        out[p + "self_attn.q_proj.weight"] = (d, d)
        out[p + "self_attn.k_proj.weight"] = (kv, d)
        out[p + "self_attn.v_proj.weight"] = (kv, d)
        out[p + "self_attn.o_proj.weight"] = (d, d)
        out[p + "mlp.gate_proj.weight"] = (h, d)
        out[p + "mlp.up_proj.weight"] = (h, d)
        out[p + "mlp.down_proj.weight"] = (d, h)
    out["model.embed_tokens.weight"] = (c["vocab_size"], d)
    out["lm_head.weight"] = (c["vocab_size"], d)
    out["model.norm.weight"] = (d,)
    out["model.norm.bias"] = (d,)
    return out


def _q8_0_torch(x):
    import torch
    rows, cols = x.shape
    b = x.reshape(rows, cols // 32, 32)
    d = b.abs().amax(-1) / 127
    inv = torch.where(d == 0, torch.zeros_like(d), 1.0 / d)
    q = torch.round(b * inv[..., None]).clamp_(-127, 127).to(torch.int8)
    out = torch.empty(rows, cols // 32, 34, dtype=torch.uint8, device=x.device)
    out[..., :2] = d.to(torch.float16).view(torch.uint8).reshape(rows, cols // 32, 2)
    out[..., 2:] = q.view(torch.uint8)
    return out.reshape(-1)


def _q6_k_torch(x):
    """Q6_K super-blocks of 256 values (the layout quant_k.go:47-62 decodes):
    ql[128] low nibbles, qh[64] high bit pairs, 16 int8 group scales, f16 d;
    value = d * scale[group] * (q - 32). Any valid encoding serves: both the
    library and the oracle decode these same bytes."""
    import torch
    rows, cols = x.shape
    b = x.reshape(-1, 16, 16)                                    # [blocks, group, 16]
    gs = b.abs().amax(-1) / 31.0                                 # group scale in weight units
    d = (gs.amax(-1) / 127.0).to(torch.float16).float()          # [blocks]
    inv_d = torch.where(d == 0, torch.zeros_like(d), 1.0 / d)
    sc = torch.round(gs * inv_d[:, None]).clamp_(-128, 127)      # int8 group scales
    step = d[:, None] * sc                                       # [blocks, group]
    inv = torch.where(step == 0, torch.zeros_like(step), 1.0 / step)
    q = (torch.round(b * inv[..., None]) + 32).clamp_(0, 63).to(torch.int32).reshape(-1, 256)
    n = q.shape[0]
    out = torch.empty(n, 210, dtype=torch.uint8, device=x.device)
    for h in range(2):
        sub = q[:, h * 128:(h + 1) * 128]
        lo, hi = sub & 15, sub >> 4
        out[:, h * 64:(h + 1) * 64] = (lo[:, :64] | (lo[:, 64:] << 4)).to(torch.uint8)
        out[:, 128 + h * 32:128 + (h + 1) * 32] = (hi[:, :32] | (hi[:, 32:64] << 2) | (hi[:, 64:96] << 4)
                                                    | (hi[:, 96:] << 6)).to(torch.uint8)
    out[:, 192:208] = sc.to(torch.int8).view(torch.uint8)
    out[:, 208:210] = d.to(torch.float16).view(torch.uint8).reshape(n, 2)
    return out.reshape(-1)


def _q5_k_torch(x):
    """Q5_K super-blocks of 256 values (the layout quant_k.go:63-85 decodes):
    f16 d and dmin, twelve bytes of packed 6-bit group scales and minima,
    qh[32] fifth bits, qs[128] nibbles; value = d * sc * q - dmin * mn."""
    import torch
    b = x.reshape(-1, 8, 32)                                     # [blocks, group, 32]
    lo = torch.clamp(b.amin(-1), max=0.0)                        # group minimum (<= 0)
    gs = (b.amax(-1) - lo) / 31.0
    d = (gs.amax(-1) / 63.0).to(torch.float16).float()
    dmin = ((-lo).amax(-1) / 63.0).to(torch.float16).float()
    inv_d = torch.where(d == 0, torch.zeros_like(d), 1.0 / d)
    inv_m = torch.where(dmin == 0, torch.zeros_like(dmin), 1.0 / dmin)
    sc = torch.round(gs * inv_d[:, None]).clamp_(0, 63)
    mn = torch.round(-lo * inv_m[:, None]).clamp_(0, 63)
    step = d[:, None] * sc
    inv = torch.where(step == 0, torch.zeros_like(step), 1.0 / step)
    q = torch.round((b + (dmin[:, None] * mn)[..., None]) * inv[..., None]).clamp_(0, 31).to(torch.int32)
    sc, mn = sc.to(torch.int32), mn.to(torch.int32)
    n = q.shape[0]
    out = torch.empty(n, 176, dtype=torch.uint8, device=x.device)
    out[:, 0:2] = d.to(torch.float16).view(torch.uint8).reshape(n, 2)
    out[:, 2:4] = dmin.to(torch.float16).view(torch.uint8).reshape(n, 2)
    out[:, 4:8] = (sc[:, :4] | ((sc[:, 4:] >> 4) << 6)).to(torch.uint8)
    out[:, 8:12] = (mn[:, :4] | ((mn[:, 4:] >> 4) << 6)).to(torch.uint8)
    out[:, 12:16] = ((sc[:, 4:] & 15) | ((mn[:, 4:] & 15) << 4)).to(torch.uint8)
    qh = torch.zeros(n, 32, dtype=torch.int32, device=x.device)
    for g in range(8):
        qh |= ((q[:, g] >> 4) & 1) << g
    out[:, 16:48] = qh.to(torch.uint8)
    for p in range(4):
        out[:, 48 + p * 32:48 + (p + 1) * 32] = ((q[:, 2 * p] & 15) | ((q[:, 2 * p + 1] & 15) << 4)).to(torch.uint8)
    return out.reshape(-1)


def synth_stablelm(config=None, dtype="Q8_0", seed=0, std=0.02, device="cpu"):
    """Returns {name: (dtype, shape, numpy uint8 payload)} for a random model.

    device selects where torch draws and encodes the weights ("cuda" is much
    faster for the 3B shape); the payload always ends in host memory."""
    import torch
    c = dict(CLIO_3B if config is None else config)
    out = {}
    names = stablelm_layer_names(c)
    shp = shapes(c)
    for idx, name in enumerate(names):
        s = shp[name]
        if len(s) == 1:
            v = np.ones(s, np.float32) if name.endswith("weight") else np.zeros(s, np.float32)
            out[name] = ("F32", s, v.view(np.uint8))
            continue
        g = torch.Generator(device=device)
        g.manual_seed(int(seed) * 1000003 + idx)
        x = torch.randn(s, generator=g, device=device, dtype=torch.float32) * std
        if dtype == "Q8_0":
            payload = _q8_0_torch(x)
        elif dtype == "Q6_K":
            payload = _q6_k_torch(x)
        elif dtype == "Q5_K":
            payload = _q5_k_torch(x)
        elif dtype == "BF16":
            payload = x.to(torch.bfloat16).view(torch.int16).view(torch.uint8).reshape(-1)
        elif dtype == "F32":
            payload = x.view(torch.uint8).reshape(-1)
        else:
            raise ValueError(f"unsupported synthetic dtype {dtype}")
        out[name] = (dtype, s, payload.cpu().numpy())
        del x, payload
    return c, out


def prompt_ids(n, vocab, seed=0, low=3):
    """n token ids uniform in [low, vocab), as the benchmark configurations draw them."""
    return np.random.default_rng(seed).integers(low, vocab, size=n, dtype=np.int64).astype(np.int32)
