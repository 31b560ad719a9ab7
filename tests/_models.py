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
