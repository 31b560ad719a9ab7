"""Shared helpers: build the oracle and the device model from one checkpoint
and run greedy decodes on both."""
import numpy as np

import oracle


def oracle_model(checkpoint, kv_dtype=np.float32, attn_splits=16):
    config = checkpoint.config
    layers = []
    for index in range(int(config["num_hidden_layers"])):
        parts = checkpoint.layer(index)
        layers.append(oracle.OracleLayer(*[oracle.OracleProjection(*p) for p in parts[:4]], *parts[4:]))
    return oracle.OracleQwen(config, layers, checkpoint.embedding, checkpoint.embedding_scales,
                             checkpoint.norms["model.norm.weight"], kv_dtype=kv_dtype,
                             attn_splits=attn_splits)


def oracle_decode(model, prompt, steps, teacher=None):
    """Prefill token by token, then `steps` greedy tokens. With `teacher`,
    the fed tokens come from it (so both sides see the same inputs) while
    the greedy choices are still recorded. Returns (logits[n], greedy[steps])."""
    state = model.new_state(len(prompt) + steps)
    logits = [model.forward_token(int(t), state).copy() for t in prompt]
    greedy = []
    for step in range(steps):
        greedy.append(int(np.argmax(logits[-1])))
        fed = greedy[-1] if teacher is None else int(teacher[step])
        logits.append(model.forward_token(fed, state).copy())
    return np.stack(logits), greedy


def oracle_for(checkpoint, cuda_model, kv_dtype=None, attn_splits=None):
    """The oracle that repeats `cuda_model`'s KV precision and attention split choice."""
    kv = kv_dtype if kv_dtype is not None else (np.float16 if cuda_model.kv_dtype == "float16" else np.float32)
    rule = cuda_model.attention_split_rule()
    if cuda_model.mode == "chain" and attn_splits is not None:
        rule = attn_splits
    return oracle_model(checkpoint, kv_dtype=kv, attn_splits=rule)


def cuda_decode(model, prompt, steps, teacher=None, attn_splits=None):
    state = model.new_state(len(prompt) + steps, attn_splits=attn_splits)
    logits = [model.forward_token(int(t), state).cpu().numpy().copy() for t in prompt]
    greedy = []
    for step in range(steps):
        greedy.append(int(np.argmax(logits[-1])))
        fed = greedy[-1] if teacher is None else int(teacher[step])
        logits.append(model.forward_token(fed, state).cpu().numpy().copy())
    state.close()
    return np.stack(logits), greedy


def top2_margin(logits):
    part = np.partition(logits, -2, axis=-1)
    return part[..., -1] - part[..., -2]


def write_lattice_checkpoint(path, config, seed=0, blocksize=64):
    """A seeded LATTICE checkpoint file (torch.save of the reference's state
    layout) for `config`: per projection the packed fields plus an
    orthogonal rotation pair, the fp32 embedding and fp32 norms. Returns the
    state dict as numpy arrays."""
    import torch

    from harsh4b_b200.cache import norm_names, projection_names
    from oracle.lattice import orthogonal, synthetic_projection

    rng = np.random.default_rng([seed, 0x1A771CE])
    hidden, inter = int(config["hidden_size"]), int(config["intermediate_size"])
    q = int(config["num_attention_heads"]) * int(config["head_dim"])
    kv = int(config["num_key_value_heads"]) * int(config["head_dim"])
    shapes = {"q_proj": (q, hidden), "k_proj": (kv, hidden), "v_proj": (kv, hidden), "o_proj": (hidden, q),
              "gate_proj": (inter, hidden), "up_proj": (inter, hidden), "down_proj": (hidden, inter)}

    def factors(width):
        dl = int(np.sqrt(width))
        while width % dl:
            dl -= 1
        return dl, width // dl

    state, plain = {}, {}
    names = projection_names(config)
    for name in names:
        rows, width = shapes[name.rsplit(".", 1)[1]]
        packed = synthetic_projection(rng, rows, width, blocksize)
        dl, dr = factors(width)
        left, right = orthogonal(rng, dl), orthogonal(rng, dr)
        plain[name] = (packed, left, right)
        state[name + ".weight"] = {k: (torch.from_numpy(np.ascontiguousarray(v)) if isinstance(v, np.ndarray) else v)
                                   for k, v in packed.items()}
        state[name + ".L"], state[name + ".R"] = torch.from_numpy(left), torch.from_numpy(right)
    embedding = (rng.standard_normal((int(config["vocab_size"]), hidden)) * 0.05).astype(np.float32)
    state["model.embed_tokens.weight"] = torch.from_numpy(embedding)
    norms = {}
    for name in norm_names(config):
        size = int(config["head_dim"]) if ("q_norm" in name or "k_norm" in name) else hidden
        norms[name] = (1.0 + 0.02 * rng.standard_normal(size)).astype(np.float32)
        state[name] = torch.from_numpy(norms[name])
    state["__latmeta__"] = {"n_linears": len(names), "encoding": "synthetic"}
    torch.save(state, str(path))
    return plain, embedding, norms
