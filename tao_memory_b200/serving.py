"""Serving-side caller of the streaming operator.

* ``RequestStates``: one request's ``StreamCache`` per layer (the operator keeps one
  state per request AND layer, and a state is never shared between concurrent
  requests or layers: reference docs/usage.md:17-20,37).
* ``save_snapshot`` / ``load_snapshot``: the export dictionaries of every layer of a
  request (reference ``StreamCache.export`` / ``from_export``, tao_stream.py:853-912)
  in one file written with ``torch.save`` and read back with
  ``torch.load(weights_only=True)``: tensors, numbers, strings and containers only,
  no pickled code.  A snapshot is still not a trust boundary (the reference's
  SECURITY.md): load only snapshots this process family wrote.
* ``DecodeScheduler``: continuous batching of decode steps over many requests of one
  model.  Requests join (after their prompts are prefilled) and leave between
  tokens; every layer's step of a token runs all active requests in one
  ``tao_attention_decode_batch`` launch set (chunks of at most ``max_batch``).

Everything here is host bookkeeping over the library's state objects; the compute is
the decode and prefill kernels of ``libtao_b200.so``.
"""

import os

import torch

from .config import TaoConfig
from .operator import new_state, tao_attention_decode_batch, tao_attention_prefill
from .stream import StreamCache

SNAPSHOT_FORMAT = 1
_SNAPSHOT_KIND = "tao_memory_b200.request"


class RequestStates:
    """One request's streaming states, one ``StreamCache`` per layer (layer l has
    ``layer_index == l``, which sets its route refresh stagger)."""

    def __init__(self, num_layers=None, config=None, states=None):
        if states is None:
            if num_layers is None or num_layers <= 0:
                raise ValueError("num_layers must be a positive integer")
            config = TaoConfig() if config is None else config
            states = [new_state(layer, config) for layer in range(num_layers)]
        states = list(states)
        if not states:
            raise ValueError("a request has at least one layer")
        if len({id(s) for s in states}) != len(states):
            raise ValueError("every layer of a request has its own state")
        for layer, st in enumerate(states):
            if not getattr(st, "is_tao_stream", False):
                raise TypeError("RequestStates holds StreamCache objects")
            if st.layer_index != layer:
                raise ValueError(f"layer {layer} holds a state with layer_index {st.layer_index}")
        self.layers = states

    def __len__(self):
        return len(self.layers)

    def __getitem__(self, layer):
        return self.layers[layer]

    @property
    def positions(self):
        """Cursor of every layer (equal between tokens of a request served layer by layer)."""
        return [st.position for st in self.layers]

    def export(self):
        """Owned tensors of every layer (see ``StreamCache.export``)."""
        return {"kind": _SNAPSHOT_KIND, "format": SNAPSHOT_FORMAT,
                "layers": [st.export() for st in self.layers]}

    @classmethod
    def from_export(cls, saved, device=None):
        """Independent states at the same cursors; execution resources are rebuilt
        from the real subsequent queries (``StreamCache.from_export``)."""
        _check_snapshot(saved)
        return cls(states=[StreamCache.from_export(layer, device=device) for layer in saved["layers"]])

    def release_execution(self, reason="request_end"):
        for st in self.layers:
            st.release_execution(reason)

    def reset(self):
        for st in self.layers:
            st.reset()

    def bytes(self):
        """``StreamCache.bytes`` of every layer, and the integer byte counts summed
        over layers."""
        per_layer = [st.bytes() for st in self.layers]
        total = {}
        for entry in per_layer:
            for key, value in entry.items():
                if key.endswith("_bytes") and isinstance(value, int) and not isinstance(value, bool):
                    total[key] = total.get(key, 0) + value
        return {"layers": per_layer, "total": total}


def _check_snapshot(saved):
    if not isinstance(saved, dict) or saved.get("kind") != _SNAPSHOT_KIND:
        raise ValueError("not a request snapshot written by save_snapshot")
    if saved.get("format") != SNAPSHOT_FORMAT:
        raise ValueError(f"snapshot format {saved.get('format')} is not {SNAPSHOT_FORMAT}")
    layers = saved.get("layers")
    if not isinstance(layers, list) or not layers:
        raise ValueError("snapshot holds no layers")
    for layer, entry in enumerate(layers):
        if not isinstance(entry, dict) or entry.get("layer_index") != layer:
            raise ValueError(f"snapshot layer {layer} is malformed")


def save_snapshot(request, path):
    """Write ``request`` (``RequestStates``, or a single ``StreamCache`` taken as a
    one-layer request) to ``path``; the file is replaced atomically."""
    if getattr(request, "is_tao_stream", False):
        request = RequestStates(states=[request]) if request.layer_index == 0 else None
        if request is None:
            raise ValueError("a single state is saved as a one-layer request only at layer_index 0")
    saved = request.export()
    tmp = f"{path}.tmp{os.getpid()}"
    torch.save(saved, tmp)
    os.replace(tmp, path)


def load_snapshot(path, device=None):
    """Read a snapshot written by ``save_snapshot`` (``torch.load`` with
    ``weights_only=True``) and rebuild its states on ``device``."""
    saved = torch.load(path, map_location="cpu", weights_only=True)
    return RequestStates.from_export(saved, device=device)


class DecodeScheduler:
    """Continuous batching of decode steps over the requests of one model.

    The model drives it token by token and layer by layer: for each token it calls
    ``decode(layer, ...)`` for layer 0, 1, ..., L-1 with the stacked [R, 1, H, D]
    operands of the active requests (row order = ``active``).  Requests join with
    ``add`` once their prompts are prefilled (``prefill``) and leave with ``remove``;
    both take effect at the next layer-0 step, so every layer of a token sees the
    same batch.  ``fusion_a`` / ``fusion_b`` are per-layer lists of [H, D, 3]
    tensors (or one [L, H, D, 3] tensor), ``alpha`` a float or a per-layer list.
    """

    def __init__(self, num_layers, fusion_a, fusion_b, alpha, max_batch=None):
        if num_layers <= 0:
            raise ValueError("num_layers must be positive")
        self.num_layers = num_layers
        self.fa = [fusion_a[i] for i in range(num_layers)]
        self.fb = [fusion_b[i] for i in range(num_layers)]
        self.alpha = [float(alpha)] * num_layers if isinstance(alpha, (int, float)) else [float(a) for a in alpha]
        if len(self.alpha) != num_layers:
            raise ValueError("alpha takes one value per layer")
        if max_batch is not None and max_batch <= 0:
            raise ValueError("max_batch must be positive")
        self.max_batch = max_batch
        self.requests = {}      # request id -> RequestStates
        self.active = []        # request ids of the current token's batch, in row order
        self._joining = []
        self._leaving = set()
        self._next_layer = 0    # the layer the current token expects next

    # -- membership ------------------------------------------------------
    def add(self, rid, request):
        """Register a request (``RequestStates`` with one state per layer); it
        joins the batch at the next token."""
        if rid in self.requests:
            raise ValueError(f"request {rid!r} is already scheduled")
        if len(request) != self.num_layers:
            raise ValueError(f"request {rid!r} has {len(request)} layers, the model {self.num_layers}")
        self.requests[rid] = request
        self._joining.append(rid)

    def remove(self, rid):
        """Take a request out after the current token; returns its states."""
        if rid not in self.requests:
            raise KeyError(rid)
        if rid in self._joining:
            self._joining.remove(rid)
            return self.requests.pop(rid)
        self._leaving.add(rid)
        return self.requests[rid]

    def _start_token(self):
        for rid in self._leaving:
            self.active.remove(rid)
            self.requests.pop(rid).release_execution()
        self._leaving.clear()
        self.active.extend(self._joining)
        self._joining.clear()
        positions = {rid: self.requests[rid].positions for rid in self.active}
        for rid, pos in positions.items():
            if len(set(pos)) != 1:
                raise RuntimeError(f"request {rid!r} has layers at different positions {pos}")

    # -- work ------------------------------------------------------------
    def prefill(self, rid, layer, q, k, v, raw_q, raw_k):
        """Prefill one layer of a request's prompt chunk ([1, T, H, D]); returns the
        layer's attention output."""
        st = self.requests[rid][layer]
        out, _ = tao_attention_prefill(q, k, v, raw_q=raw_q, raw_k=raw_k, fusion_a=self.fa[layer],
                                       fusion_b=self.fb[layer], alpha=self.alpha[layer], state=st,
                                       position=st.position)
        return out

    def decode(self, layer, q, k, v, raw_q, raw_k, out=None):
        """One token of ``layer`` for every active request: operands [R, 1, H, D]
        in ``active`` order (R = len(active) after the membership changes, which
        apply at layer 0).  Returns the [R, 1, H, D] output."""
        if layer != self._next_layer:
            raise RuntimeError(f"layer {layer} called while the token expects layer {self._next_layer}")
        if layer == 0:
            self._start_token()
        if not self.active:
            raise RuntimeError("no active request")
        r = len(self.active)
        if q.shape[0] != r:
            raise ValueError(f"operands carry {q.shape[0]} rows for {r} active requests")
        states = [self.requests[rid][layer] for rid in self.active]
        step = self.max_batch or r
        if out is None:
            out = torch.empty_like(q) if q.device.type != "cpu" else torch.empty(q.shape, dtype=q.dtype).pin_memory()
        for lo in range(0, r, step):
            hi = min(r, lo + step)
            tao_attention_decode_batch(q[lo:hi], k[lo:hi], v[lo:hi], raw_q=raw_q[lo:hi], raw_k=raw_k[lo:hi],
                                       fusion_a=self.fa[layer], fusion_b=self.fb[layer],
                                       alpha=self.alpha[layer], states=states[lo:hi], out=out[lo:hi])
        self._next_layer = (layer + 1) % self.num_layers
        return out
