"""Seeded synthetic DiT checkpoints for tests and benchmarks (no model files are involved).

Tensor names and shapes are the ones dit_block / dit_head / dit_tail read (src/dit.h:164-323),
shaped as PyTorch [out][in] (= ggml [in, out]); 1-D tensors are vectors.  Weights are drawn from
N(0, std) (BASELINE: std 0.02), norms' gammas near 1, biases and adaLN offsets small.
"""
import numpy as np

MEDIUM_LIKE = dict(io=64, dim=1536, depth=24, heads=24, head_dim=64, cond_dim=768, mem_tokens=64, rot=32,
                   time_dim=256, ff_inner=6144, differential=0, rope_base=10000.0, norm_eps=1e-5, qk_eps=1e-6,
                   time_min_freq=0.5, time_max_freq=10000.0)


def tensor_shapes(cfg):
    """name -> shape ([out, in] for weights, [n] for vectors, [mem, dim] for memory tokens)."""
    D, io, cd, td, I = cfg["dim"], cfg["io"], cfg["cond_dim"], cfg["time_dim"], cfg["ff_inner"]
    qkv = (5 if cfg["differential"] else 3) * D
    s = {
        "dit.time_embed.0.weight": (D, td), "dit.time_embed.0.bias": (D,),
        "dit.time_embed.2.weight": (D, D), "dit.time_embed.2.bias": (D,),
        "dit.global_embed.0.weight": (D, cd), "dit.global_embed.2.weight": (D, D),
        "dit.gce.0.weight": (D, D), "dit.gce.0.bias": (D,),
        "dit.gce.2.weight": (6 * D, D), "dit.gce.2.bias": (6 * D,),
        "dit.cond_embed.0.weight": (D, cd), "dit.cond_embed.2.weight": (D, D),
        "dit.pre_conv.weight": (io, io), "dit.proj_in.weight": (D, io),
        "dit.proj_out.weight": (io, D), "dit.post_conv.weight": (io, io),
        "dit.memory_tokens": (cfg["mem_tokens"], D),
    }
    for l in range(cfg["depth"]):
        p = f"dit.{l}."
        s.update({
            p + "ssg": (6 * D,), p + "pre_norm.gamma": (D,),
            p + "self.qkv.weight": (qkv, D), p + "self.q_norm.gamma": (64,), p + "self.k_norm.gamma": (64,),
            p + "self.out.weight": (D, D), p + "cross_norm.gamma": (D,),
            p + "cross.q.weight": ((2 if cfg["differential"] else 1) * D, D),
            p + "cross.kv.weight": ((3 if cfg["differential"] else 2) * D, D),
            p + "cross.q_norm.gamma": (64,), p + "cross.k_norm.gamma": (64,),
            p + "cross.out.weight": (D, D), p + "ff_norm.gamma": (D,),
            p + "ff.proj.weight": (2 * I, D), p + "ff.proj.bias": (2 * I,),
            p + "ff.out.weight": (D, I), p + "ff.out.bias": (D,),
        })
        if cfg.get("local_dim", 0):   # inpaint local conditioning (src/dit.h:246-254)
            s.update({p + "local.0.weight": (D, cfg["local_dim"]), p + "local.0.bias": (D,),
                      p + "local.2.weight": (D, D), p + "local.2.bias": (D,)})
    return s


def is_weight(name):
    return name.endswith(".weight")


def synth_tensor(name, shape, rng, std):
    if is_weight(name):
        return rng.normal(0.0, std, shape).astype(np.float32)
    if name.endswith("gamma"):
        return (1.0 + 0.1 * rng.standard_normal(shape)).astype(np.float32)
    if name.endswith("memory_tokens"):
        return rng.standard_normal(shape).astype(np.float32)
    return (0.05 * rng.standard_normal(shape)).astype(np.float32)   # biases, ssg


def default_targets(cfg):
    """DoRA targets of BASELINE config 4: q/k/v (fused qkv), o and both MLP projections."""
    names = []
    for l in range(cfg["depth"]):
        names += [f"dit.{l}.self.qkv.weight", f"dit.{l}.self.out.weight", f"dit.{l}.ff.proj.weight",
                  f"dit.{l}.ff.out.weight"]
    return names


def scope_targets(cfg, scope):
    """Adapter targets of a LoRA scope, sorted by name like the reference's target enumeration
    (src/train_lora.h:54-117): "full" = every 2-D `dit.*.weight` (the 7 per-block projections and
    the 12 head / tail linears; this DiT has no inpaint `local.*` weights), "core" = the per-block
    projections only, "config4" = default_targets."""
    if scope == "config4":
        return default_targets(cfg)
    names = [n for n, shp in tensor_shapes(cfg).items() if is_weight(n) and len(shp) == 2]
    if scope == "core":
        names = [n for n in names if n[4:5].isdigit()]
    elif scope != "full":
        raise ValueError(f"unknown scope {scope}")
    return sorted(names)
