"""Functional Tao attention on B200: the reference's public API, drop-in.

Reference: tao_attention/operator.py:42-137 (``tao_attention``, ``new_state``,
``tao_attention_prefill``, ``tao_attention_decode``).  Inputs are
[batch, tokens, heads, width]; ``raw_q``/``raw_k`` are the projections before the
caller's Q/K transform, ``q``/``k`` the local-attention operands after it.  The
streaming calls take batch 1, bf16, width 64 or 128 (the reference's documented
envelope) and mutate and return the state.

Added beyond the reference: ``tao_attention_decode_batch`` advances many
independent requests by one token each in one set of kernel launches.
"""

import torch

from .config import TaoConfig
from .stream import StreamCache, run_batch, run_batch_host, WINDOW

DEFAULT_CONFIG = TaoConfig()


def new_state(layer_index, config=DEFAULT_CONFIG):
    """Independent mutable per-request, per-layer inference state (operator.py:57-60)."""
    return StreamCache(layer_index, route_interval=2, fusion_mode="pointwise",
                       fused_fine=True, config=config)


def _check_local_flash(local_flash):
    if local_flash is not None:
        raise ValueError("local_flash callbacks are not supported: local attention runs in "
                         "the library's own sm_100a kernel")


def tao_attention_prefill(q, k, v, *, raw_q, raw_k, fusion_a, fusion_b, alpha,
                          state, position, local_flash=None):
    """Advance only the supplied new tokens; reads happen before each 768 seal.

    Raises ValueError when ``position`` differs from the state's cursor
    (operator.py:77-78).  Returns (output [1, T, H, D], state).
    """
    if position != state.position:
        raise ValueError("position must match this request's causal cursor")
    _check_local_flash(local_flash)
    if q.dim() != 4 or q.shape[0] != 1:
        raise ValueError("streaming calls take [1, tokens, heads, width] operands")
    tokens = q.shape[1]
    out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    start = 0
    with torch.no_grad():
        while start < tokens:
            width = state.next_chunk(tokens - start)
            sl = slice(start, start + width)
            state._run(q[:, sl], k[:, sl], v[:, sl], raw_q[:, sl], raw_k[:, sl],
                       fusion_a, fusion_b, alpha, out[:, sl])
            start += width
    return out, state


def tao_attention_decode(q, k, v, *, raw_q, raw_k, fusion_a, fusion_b, alpha,
                         state, position, local_flash=None):
    """One-token prefill (operator.py:130-137)."""
    if q.shape[1] != 1:
        raise ValueError("decode accepts exactly one new query/key/value")
    return tao_attention_prefill(q, k, v, raw_q=raw_q, raw_k=raw_k, fusion_a=fusion_a,
                                 fusion_b=fusion_b, alpha=alpha, state=state,
                                 position=position, local_flash=local_flash)


def tao_attention_decode_batch(q, k, v, *, raw_q, raw_k, fusion_a, fusion_b, alpha,
                               states, positions=None, out=None):
    """Decode one token for each of ``len(states)`` independent requests.

    q, k, v, raw_q, raw_k: [R, 1, H, D] bf16 (row r belongs to states[r]); all
    states share fusion_a/fusion_b/alpha (one layer's parameters).  Each state
    advances by one; the result equals R separate ``tao_attention_decode`` calls.
    The operands may be page-locked host tensors: the library then moves them in
    and the result out itself (in the same captured step for graph-configured
    states) and returns a page-locked host tensor, valid after the current stream
    is synchronised.
    """
    if q.dim() != 4 or q.shape[1] != 1 or q.shape[0] != len(states):
        raise ValueError("batched decode takes [len(states), 1, heads, width] operands")
    if positions is not None:
        for st, p in zip(states, positions):
            if p != st.position:
                raise ValueError("position must match this request's causal cursor")
    if len({id(s) for s in states}) != len(states):
        raise ValueError("a state may appear only once per batch")
    if q.device.type == "cpu":
        # operands in page-locked host memory: the result goes to page-locked host
        # memory too, valid once the device's current stream has reached the step
        if out is None:
            out = torch.empty(q.shape, dtype=q.dtype).pin_memory()
        with torch.no_grad():
            run_batch_host(list(states), (q, k, v, raw_q, raw_k), fusion_a, fusion_b, alpha, out)
        return out, states
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    with torch.no_grad():
        run_batch(list(states), q, k, v, raw_q, raw_k, fusion_a, fusion_b, alpha, out)
    return out, states


def tao_attention(q, k, v, *, raw_q, raw_k, fusion_a, fusion_b, alpha,
                  config=DEFAULT_CONFIG, local_flash=None):
    """Full differentiable sequence read with fresh routing at every query
    (operator.py:42-54).  ``alpha`` may be a float or a per-head sequence."""
    _check_local_flash(local_flash)
    from .training import tao_attention_train
    return tao_attention_train(q, k, v, raw_q, raw_k, fusion_a, fusion_b, alpha, config)


__all__ = ["new_state", "tao_attention", "tao_attention_prefill", "tao_attention_decode",
           "tao_attention_decode_batch", "StreamCache", "WINDOW"]
