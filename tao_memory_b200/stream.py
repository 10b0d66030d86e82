"""Device-resident per-request, per-layer Tao state (reference ``StreamCache``).

Reference: tao_attention/tao_stream.py:790-1094 (StreamCache) and 126-527
(LayerState).  The semantic content is the same (exact local window, sealed fine
matrices and log-partitions, pages, selected route ids, cursor) but it lives in
fixed-capacity device buffers described by one ``TaoState`` descriptor:

* the local window is a 768-slot ring (slot = position % 768) for k, v and raw k,
  so no per-token concatenation happens;
* fine matrices are appended in place into a preallocated bank that doubles when
  full, instead of the reference's ``torch.cat`` repack at every seal;
* the page-normalisation memo (page log-partitions and their softmax over pages)
  is refreshed by the seal kernel, on the device.

``export()``/``from_export()`` use the reference's snapshot dictionary, so
snapshots move between the two implementations.
"""

import ctypes
import math
import weakref

import torch

from . import _lib
from .config import TaoConfig, routed_counts

WINDOW, FINE, KEEP, GROUP = 768, 256, 512, 8
ROUTE_CAP = 256
MIN_CAP = 64          # initial fine-bank capacity (fines); doubles when full
WRITERS_B200 = ("softmax", "regularized_association", "feature_mass_association", "structured_gram_association")
# writers whose fines are read with the feature-mass mixture (tao_stream.py:362-367)
FEATURE_WRITERS = ("feature_mass_association", "structured_gram_association")
_BF16 = torch.bfloat16
TRAIN_COARSE = True    # the training path's coarse value branch (tao_memory_b200.training_coarse)


def window_start(pos):
    """First absolute position of the exact local window while serving ``pos``."""
    return 0 if pos < WINDOW else FINE * ((pos - KEEP) // FINE)


def sealed_at(pos):
    """Sealed fines before the token at ``pos`` is processed."""
    return (pos - WINDOW) // FINE + 1 if pos >= WINDOW else 0


def is_refresh(pos, layer, config):
    first_turn = WINDOW + config.layer_stagger * layer
    return pos == WINDOW or (pos >= first_turn and (pos - first_turn) % config.route_period == 0)


def check_config(config, training=False):
    """The sm_100a kernels implement the index-only preset with all four fine
    writers (softmax, regularised-association, feature-mass and structured-Gram),
    in streaming and in training, and the coarse value branch (coarse_index_only=False,
    the historical default) with the softmax writer."""
    if (config.fine_tokens, config.local_keep, config.coarse_group) != (FINE, KEEP, GROUP):
        raise ValueError("kernels are specialised for fine_tokens=256, local_keep=512, coarse_group=8")
    writers = WRITERS_B200
    if config.fine_writer not in writers:
        raise NotImplementedError("fine_writer=%r is not implemented on B200 %s(implemented: %s)"
                                  % (config.fine_writer, "training " if training else "", ", ".join(writers)))
    if not config.coarse_index_only:
        if config.fine_writer != "softmax":
            raise NotImplementedError("the coarse value branch (coarse_index_only=False) is implemented on "
                                      "B200 with the softmax fine writer")
        if training and not TRAIN_COARSE:
            raise NotImplementedError("the coarse value branch is implemented on B200 for streaming")


def _structured_matrix(square, cross, mass, count):
    """C of the structured-Gram writer (structured_writer.py:17-34) on the device in
    fp32, bf16 at the end: per channel the clamped variance var = square -
    mass^2/count plus a ridge (the mean square mass) forms the diagonal; a rank-one
    term along t = var/diag (dropped when every var is zero) and the rank-one mass
    term are inverted in closed form (Sherman-Morrison, denominator count +
    mass . hm).  square, mass [1,H,D], cross [1,H,D,D]; the fp32 operations run in
    the reference's order."""
    var = (square - mass * mass / count).clamp_min(0)
    flat = var.sum(-1, keepdim=True) == 0
    ridge = square.sum(-1, keepdim=True) / mass.shape[-1]
    diag = var + ridge
    t = torch.where(flat, torch.zeros_like(var), var / diag)
    norm = torch.where(flat, torch.ones_like(ridge), (var * ridge / diag).sum(-1, keepdim=True))
    tx = (t.unsqueeze(-1) * cross).sum(-2)
    hx = cross / diag.unsqueeze(-1) + t.unsqueeze(-1) * tx.unsqueeze(-2) / norm.unsqueeze(-1)
    hm = mass / diag + t * (t * mass).sum(-1, keepdim=True) / norm
    mhx = (mass.unsqueeze(-1) * hx).sum(-2)
    den = count + (mass * hm).sum(-1, keepdim=True)
    return (hx - hm.unsqueeze(-1) * mhx.unsqueeze(-2) / den.unsqueeze(-1)).to(_BF16)


def policy_for(config):
    return _lib.TaoPolicy(FINE, KEEP, GROUP, config.route_period, config.layer_stagger,
                          config.budget_root_scale, config.budget_offset, ROUTE_CAP,
                          int(config.fine_writer in FEATURE_WRITERS), int(not config.coarse_index_only))


def _policy_key(config):
    """The configuration fields a captured or cached decode step bakes in."""
    return (config.route_period, config.layer_stagger, config.budget_root_scale, config.budget_offset,
            config.fine_writer in FEATURE_WRITERS, config.coarse_index_only)


class _Workspace:
    """Grow-only device scratch, one per (device, stream).  Calls on one stream run
    in order and share it; calls on two streams of one device get separate
    scratch, so requests decoded concurrently on different streams do not race on
    route slots, partials or the error word."""

    cache = {}

    @classmethod
    def get(cls, device, stream, nbytes):
        key = (device, stream)
        buf = cls.cache.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            cls.cache[key] = buf
        return buf

    @classmethod
    def on_device(cls, device):
        return [(stream, buf) for (dev, stream), buf in list(cls.cache.items()) if dev == device]


class StreamCache:
    """One request's one-layer exact-local and hierarchical history state."""

    is_tao_stream = True

    def __init__(self, layer_index, route_interval=2, fusion_mode="pointwise",
                 pending_coarse_elision=False, pending_coarse_mask=False,
                 fused_fine=True, config=TaoConfig()):
        check_config(config)
        self.config = config
        self.layer_index = layer_index
        self.route_interval = route_interval
        self.fusion_mode = fusion_mode
        self.fused_fine = fused_fine
        self.pending_coarse_elision = pending_coarse_elision
        self.pending_coarse_mask = pending_coarse_mask
        self.position = 0
        self.history_path_ablation = False
        self.history_value_ablation = False
        self._buf = None          # dict of device tensors
        self._graph = None        # _DecodeGraph (config.q1_history_region_graph)
        self._gram = self._cross = None  # fp32 [1,H,D,D] writer statistics (association writers)
        self._mass = None         # fp32 [1,H,D] accumulated feature mass (feature-read writers)
        self._square = None       # fp32 [1,H,D] accumulated sum u*u (structured-Gram writer)
        self._desc = None         # device TaoState (uint8 tensor)
        self._host = None         # ctypes TaoState mirror
        self._ptrs = None         # device array holding the descriptor address
        self.heads = self.width = None
        self.device = None
        self.cap_fines = 0
        self._counters = dict(fusion_pointwise_calls=0, fusion_no_history_local_returns=0,
                              fused_fine_calls=0, peak_local_tokens=0)

    # -- reference API ---------------------------------------------------
    def get_pos(self):
        return self.position

    def next_chunk(self, desired):
        """Tokens the next call may take without crossing a seal (tao_stream.py:914-917)."""
        current = self.position - window_start(self.position) if self.position else 0
        return min(desired, FINE, WINDOW - current)

    def advance(self, count):
        self.position += count

    def release_execution(self, reason="request_end"):
        """Drop execution-only resources (graphs, cached pointer arrays)."""
        self._ptrs = None
        self._graph = None

    def reset(self):
        """Discard this request's state without touching another request."""
        self.release_execution("reset")
        self.__init__(self.layer_index, self.route_interval, self.fusion_mode,
                      self.pending_coarse_elision, self.pending_coarse_mask,
                      self.fused_fine, self.config)

    # -- device buffers --------------------------------------------------
    def _allocate(self, heads, width, device, cap):
        device = torch.device(device)
        if device.type == "cuda" and device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        if width not in (64, 128):
            raise ValueError("head width must be 64 or 128")
        cap = max(GROUP, int(math.ceil(cap / GROUP)) * GROUP)
        z = lambda *shape, dt=_BF16: torch.zeros(*shape, dtype=dt, device=device)
        pages = cap // GROUP + 1
        self._buf = dict(
            k_ring=z(heads, WINDOW, width), v_ring=z(heads, WINDOW, width),
            rk_ring=z(heads, WINDOW, width),
            fine_c=z(heads, cap, width, width), fine_z=z(heads, cap, width),
            page_z=z(heads, pages, width), page_w=z(heads, pages, width),
            route_ids=z(heads, ROUTE_CAP, dt=torch.int32),
            route_pages=z(heads, ROUTE_CAP, dt=torch.int32),
            counters=z(heads, dt=torch.int32))
        if not self.config.coarse_index_only:   # coarse value branch: page matrices and page softmax
            self._buf["page_c"] = z(heads, pages, width, width)
            self._buf["coarse_w"] = z(heads, pages, width)
        self.heads, self.width, self.device, self.cap_fines = heads, width, device, cap
        h = _lib.TaoState()
        for name in ("k_ring", "v_ring", "rk_ring", "fine_c", "fine_z", "page_z", "page_w",
                     "route_ids", "route_pages", "counters", "page_c", "coarse_w"):
            if name in self._buf:
                setattr(h, name, self._buf[name].data_ptr())
        h.position = self.position
        h.cap_fines, h.route_cap, h.layer_index = cap, ROUTE_CAP, self.layer_index
        h.heads, h.width = heads, width
        self._host = h
        self._desc = torch.zeros(ctypes.sizeof(_lib.TaoState), dtype=torch.uint8, device=device)
        self._upload()
        self._ptrs = None

    def _upload(self):
        raw = bytes(self._host)
        self._desc.copy_(torch.frombuffer(bytearray(raw), dtype=torch.uint8))

    def _download(self):
        """Read the device-updated descriptor fields (synchronising)."""
        raw = self._desc.cpu().numpy().tobytes()
        ctypes.memmove(ctypes.addressof(self._host), raw, len(raw))
        return self._host

    def _grow(self, need):
        """Double the fine bank until it holds ``need`` fines (in-place append
        afterwards; existing fines are copied once)."""
        cap = self.cap_fines
        while cap < need:
            cap *= 2
        if cap == self.cap_fines:
            return
        host = self._download()
        old = self._buf
        s = sealed_at(self.position)
        p = s // GROUP + (s % GROUP > 0)
        self._allocate(self.heads, self.width, self.device, cap)
        for name in ("k_ring", "v_ring", "rk_ring", "route_ids", "route_pages"):
            self._buf[name].copy_(old[name])
        self._buf["fine_c"][:, :s].copy_(old["fine_c"][:, :s])
        self._buf["fine_z"][:, :s].copy_(old["fine_z"][:, :s])
        self._buf["page_z"][:, :p].copy_(old["page_z"][:, :p])
        self._buf["page_w"][:, :p].copy_(old["page_w"][:, :p])
        if "page_c" in old:
            self._buf["page_c"][:, :p].copy_(old["page_c"][:, :p])
            self._buf["coarse_w"][:, :p].copy_(old["coarse_w"][:, :p])
        for f in ("n_route", "n_chosen", "route_refreshes", "seal_events"):
            setattr(self._host, f, getattr(host, f))
        self._host.position = self.position
        self._upload()

    def _pointer_array(self):
        if self._ptrs is None:
            self._ptrs = torch.tensor([self._desc.data_ptr()], dtype=torch.int64, device=self.device)
        return self._ptrs

    def _ensure(self, heads, width, device, tokens):
        if device.type == "cuda" and device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        if self._buf is None:
            end = self.position + tokens
            self._allocate(heads, width, device, max(MIN_CAP, sealed_at(end) + 1))
        elif (heads, width) != (self.heads, self.width) or device != self.device:
            raise ValueError("a state serves one head count, width and device")
        need = sealed_at(self.position + tokens) + 1
        if need > self.cap_fines:
            self._grow(need)

    # -- one chunk through the kernels ------------------------------------
    def _run(self, q, k, v, raw_q, raw_k, fusion_a, fusion_b, alpha, out):
        """Advance by q.shape[1] tokens (must not cross a seal); fused output -> out."""
        if (self.config.q1_history_region_graph and self.config.fine_writer == "softmax"
                and q.shape[1] == 1 and q.device.type == "cuda"):
            _DecodeGraph.step(self, q, k, v, raw_q, raw_k, fusion_a, fusion_b, alpha, out)
        else:
            run_batch([self], q, k, v, raw_q, raw_k, fusion_a, fusion_b, alpha, out)

    # -- association fine writers (tao_stream.py:62-65, 72-74, 463-500) ---
    def _seal_writer(self, s):
        """Replace fine ``s`` (just sealed by the softmax writer kernels) by the
        regularised association matrix of the same block: statistics on the tensor
        cores (``tao_writer_stats``), the Cholesky solve in torch.linalg.  The
        block's 256 tokens are still in the ring (nothing has been appended since
        the seal).  As in the reference with index-only pages, the fp32 statistics
        accumulate without reset.

        Regularised writer: z stays the softmax writer's log-partition.  Feature-mass
        writer: z = bf16(log mass) of the block, the solve does not check the
        factorisation (association_writer.py:21-32 called unchecked), and the page
        receiving the fine gets page_z = bf16(log accumulated mass); the page weights
        are then recomputed on the device.  Structured-Gram writer: the same z and
        page z, C from the closed-form structured inverse (``_structured_matrix``)
        of the square mass (the Gram's diagonal), X and the mass; no dense Gram is
        kept."""
        heads, width = self.heads, self.width
        writer = self.config.fine_writer
        feature = writer in FEATURE_WRITERS
        slot0 = (s * FINE) % WINDOW
        gram = torch.empty(1, heads, width, width, dtype=torch.float32, device=self.device)
        cross = torch.empty_like(gram)
        mass = torch.empty(1, heads, width, dtype=torch.float32, device=self.device) if feature else None
        k = self._buf["rk_ring"][:, slot0:slot0 + FINE]
        v = self._buf["v_ring"][:, slot0:slot0 + FINE]
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(_lib.lib().tao_writer_stats(k.data_ptr(), v.data_ptr(), width, WINDOW * width, 0, 1, heads,
                                               width, gram.data_ptr(), cross.data_ptr(),
                                               None if mass is None else mass.data_ptr(), stream))
        if writer == "structured_gram_association":
            square = gram.diagonal(dim1=-2, dim2=-1).contiguous()
            c = _structured_matrix(square, cross, mass, FINE)
            self._square = square if self._square is None else self._square + square
        else:
            reg = gram.diagonal(dim1=-2, dim2=-1).sum(-1) / width
            system = gram + reg[..., None, None] * torch.eye(width, dtype=torch.float32, device=self.device)
            if feature:
                factor, _ = torch.linalg.cholesky_ex(system, check_errors=False)
            else:
                factor = torch.linalg.cholesky(system)
            c = torch.cholesky_solve(cross, factor).to(_BF16)
            self._gram = gram if self._gram is None else self._gram + gram
        self._buf["fine_c"][:, s].copy_(c[0])
        self._cross = cross if self._cross is None else self._cross + cross
        if feature:
            self._mass = mass if self._mass is None else self._mass + mass
            self._buf["fine_z"][:, s].copy_(mass[0].log().to(_BF16))
            self._buf["page_z"][:, s // GROUP].copy_(self._mass[0].log().to(_BF16))
            _lib.check(_lib.lib().tao_state_refresh_page_weights(self._desc.data_ptr(), heads, width, s + 1,
                                                                 stream))

    # -- snapshots (reference dictionary format, tao_stream.py:853-912) --
    def export(self):
        """Owned tensors for a checkpoint or an independent request."""
        s = sealed_at(self.position)
        layer = {"n_route": 0, "n_chosen": 0, "route_refreshes": 0}
        local = None
        fine_c = None
        pages, pending = [], []
        route = None
        if self._buf is not None:
            host = self._download()
            layer = {"n_route": host.n_route, "n_chosen": host.n_chosen,
                     "route_refreshes": host.route_refreshes}
            n = self.position - window_start(self.position)
            if n:
                local = tuple(self._gather_ring(name, window_start(self.position), n)
                              for name in ("k_ring", "v_ring", "rk_ring"))
            if s:
                fine_c = self._buf["fine_c"][:, :s].unsqueeze(0).clone()
                fz = self._buf["fine_z"]
                pz = self._buf["page_z"]
                pc = self._buf.get("page_c")
                for p in range(s // GROUP):
                    pages.append((pz[:, p].unsqueeze(0).clone(),
                                  None if pc is None else pc[:, p].unsqueeze(0).clone(),
                                  fz[:, p * GROUP:(p + 1) * GROUP].unsqueeze(0).clone()))
                for i in range((s // GROUP) * GROUP, s):
                    pending.append(fz[:, i].unsqueeze(0).clone())
            if host.n_route:
                ids = self._buf["route_ids"][:, :host.n_route].to(torch.int64)
                chosen = self._buf["route_pages"][:, :host.n_chosen].to(torch.int64)
                route = (chosen.view(1, 1, self.heads, -1).clone(),
                         ids.view(1, 1, self.heads, -1).clone())
        return {
            "layer_index": self.layer_index, "config": self.config.export(),
            "route_interval": self.route_interval, "fusion_mode": self.fusion_mode,
            "fused_fine": self.fused_fine, "position": self.position, "local": local,
            "packed_fine_c": fine_c, "pages": pages, "pending_z": pending,
            "pending_square_mass": None if self._square is None else self._square.clone(),
            "pending_mass": None if self._mass is None else self._mass.clone(),
            "pending_gram": None if self._gram is None else self._gram.clone(),
            "pending_cross": None if self._cross is None else self._cross.clone(),
            "route_ids": route, "route_key": None,
            "state_version": s, "route_refreshes": layer["route_refreshes"],
            "fine_seal_events": s,
        }

    @classmethod
    def from_export(cls, saved, device=None):
        """Restore the same cursor with no alias to the exported tensors.  Accepts
        dictionaries produced by this class or by the reference StreamCache."""
        state = cls(saved["layer_index"], saved["route_interval"], saved["fusion_mode"],
                    fused_fine=saved["fused_fine"], config=TaoConfig(**saved["config"]))
        pos = saved["position"]
        state.position = pos
        local = saved["local"]
        if local is None and not saved["pages"] and not saved["pending_z"]:
            return state
        sample = local[0] if local is not None else saved["packed_fine_c"]
        heads, width = sample.shape[2], sample.shape[-1]
        dev = torch.device(device) if device is not None else (
            sample.device if sample.is_cuda else torch.device("cuda", torch.cuda.current_device()))
        s = sealed_at(pos)
        state._allocate(heads, width, dev, max(64, s + 1))
        b = state._buf
        for name, attr in (("pending_gram", "_gram"), ("pending_cross", "_cross"), ("pending_mass", "_mass"),
                           ("pending_square_mass", "_square")):
            if saved.get(name) is not None:
                setattr(state, attr, saved[name].to(dev, torch.float32).clone())
        if local is not None:
            n = local[0].shape[1]
            if n != pos - window_start(pos):
                raise ValueError("snapshot local window does not match its position")
            for name, t in zip(("k_ring", "v_ring", "rk_ring"), local):
                state._scatter_ring(name, pos - n, t)
        fz = [z.reshape(heads, -1, width) for _, _, z in saved["pages"]]
        fz += [z.reshape(heads, 1, width) for z in saved["pending_z"]]
        if s:
            if sum(t.shape[1] for t in fz) != s:
                raise ValueError("snapshot fine count does not match its position")
            b["fine_z"][:, :s].copy_(torch.cat(fz, dim=1).to(dev, _BF16))
            b["fine_c"][:, :s].copy_(saved["packed_fine_c"][0].to(dev, _BF16))
        if "page_c" in b:
            for p, (_, pc, _) in enumerate(saved["pages"]):
                if pc is None:
                    raise ValueError("snapshot of a coarse-value configuration without page matrices")
                b["page_c"][:, p].copy_(pc.reshape(heads, width, width).to(dev, _BF16))
        h = state._host
        route = saved["route_ids"]
        if route is not None:
            chosen, ids = route
            m, kc = ids.shape[-1], chosen.shape[-1]
            b["route_ids"][:, :m].copy_(ids.reshape(heads, m).to(dev, torch.int32))
            b["route_pages"][:, :kc].copy_(chosen.reshape(heads, kc).to(dev, torch.int32))
            h.n_route, h.n_chosen = m, kc
        h.route_refreshes = saved.get("route_refreshes", 0)
        h.seal_events = s
        h.position = pos
        state._upload()
        stream = torch.cuda.current_stream(dev).cuda_stream
        if state.config.fine_writer in FEATURE_WRITERS and s:
            # page_z is not a function of fine_z for this writer: completed pages keep
            # the snapshot's values, the pending page is bf16(log accumulated mass)
            for p, (pz, _, _) in enumerate(saved["pages"]):
                b["page_z"][:, p].copy_(pz.reshape(heads, width).to(dev, _BF16))
            if s % GROUP:
                if state._mass is None:
                    raise ValueError("feature-mass snapshot with pending fines has no pending_mass")
                b["page_z"][:, s // GROUP].copy_(state._mass[0].log().to(_BF16))
            _lib.check(_lib.lib().tao_state_refresh_page_weights(state._desc.data_ptr(), heads, width, s, stream))
        else:
            _lib.check(_lib.lib().tao_state_rebuild_memo(state._desc.data_ptr(), heads, width, s, stream))
        return state

    def _gather_ring(self, name, first, count):
        out = torch.empty(1, count, self.heads, self.width, dtype=_BF16, device=self.device)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(_lib.lib().tao_ring_gather(self._buf[name].data_ptr(), self.heads, self.width,
                                              first, count, out.data_ptr(), stream))
        return out

    def _scatter_ring(self, name, first, t):
        t = t.to(self.device, _BF16).contiguous()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(_lib.lib().tao_ring_scatter(self._buf[name].data_ptr(), self.heads, self.width,
                                               first, t.shape[1], t.data_ptr(), stream))

    def bytes(self):
        """Byte accounting with the reference's key names (tao_stream.py:988-1094)."""
        s = sealed_at(self.position)
        heads, width = self.heads or 0, self.width or 0
        pages, pending = s // GROUP, s % GROUP
        history = (pages * (GROUP + 1) + pending) * (width * width + width) * heads * 2
        if self.config.coarse_index_only:
            history -= pages * width * width * heads * 2  # index-only pages hold no matrix
        local = self.position - window_start(self.position)
        logical_local = local * 2 * heads * width * 2
        physical = 0 if self._buf is None else sum(t.numel() * t.element_size() for t in self._buf.values())
        n_route = 0 if self._buf is None else self._download().n_route
        route_bytes = n_route * heads * 8
        stat = lambda t: 0 if t is None else t.numel() * t.element_size()
        gram_cross = stat(self._gram) + stat(self._cross)
        return {"history_bytes": history, "page_normalization_memo_bytes": 0,
                "pending_writer_bytes": gram_cross + stat(self._mass) + stat(self._square),
                "pending_gram_cross_bytes": gram_cross,
                "pending_cross_bytes": stat(self._cross), "pending_square_mass_bytes": stat(self._square),
                "pending_feature_mass_bytes": stat(self._mass), "fused_fine": self.fused_fine,
                "fusion_mode": self.fusion_mode, "fine_seal_events": s,
                "route_integer_bytes": route_bytes,
                "logical_local_bf16_kv_bytes": logical_local,
                "logical_retained_bytes": history + logical_local,
                "physical_local_including_raw_key_bytes": local * 3 * heads * width * 2,
                "unique_allocated_cache_storage_bytes": physical,
                "local_length_tokens": local, "completed_coarse_pages": pages,
                "pending_fine_states": pending,
                "selected_fine_per_layer": [n_route],
                "fine_matrix_repack_bytes": 0, **self._counters}


def _as_bf16(t, name, device):
    if t.device != device:
        raise ValueError(f"{name} must be on {device}")
    if t.dtype != _BF16:
        raise ValueError("B200 streaming supports bfloat16 operands (the reference's documented envelope)")
    return t.contiguous()


class _BatchArgs:
    """Per-batch ctypes arguments reused across calls (pointer array, policy,
    cursor/capacity/layer arrays, workspace size)."""

    cache = {}

    def __init__(self, states, w, heads, width, dev):
        self.r = len(states)
        self.ptrs = torch.tensor([st._desc.data_ptr() for st in states], dtype=torch.int64, device=dev)
        self.policy = policy_for(states[0].config)
        self.pos = (ctypes.c_int64 * self.r)()
        self.cap = (ctypes.c_int32 * self.r)(*[st.cap_fines for st in states])
        self.layers = (ctypes.c_int32 * self.r)(*[st.layer_index for st in states])
        self.nbytes = _lib.lib().tao_stream_workspace_bytes(self.r, w, heads, width, ROUTE_CAP,
                                                           ctypes.byref(self.policy))

    @classmethod
    def get(cls, states, w, heads, width, dev):
        # everything the cached arrays hold is part of the key: a freed state's
        # descriptor address can be reused by a new state with another layer index
        key = (tuple((st._desc.data_ptr(), st.cap_fines, st.layer_index) for st in states), w, heads, width,
               _policy_key(states[0].config))
        args = cls.cache.get(key)
        if args is None:
            if len(cls.cache) > 256:
                cls.cache.clear()
            args = cls.cache[key] = cls(states, w, heads, width, dev)
        return args


def run_batch(states, q, k, v, raw_q, raw_k, fusion_a, fusion_b, alpha, out, allow_graph=True):
    """Advance every state by q.shape[1] tokens in one set of kernel launches.

    q, k, v, raw_q, raw_k, out: [len(states), tokens, H, D] bf16 on one device.
    The chunk must not cross a seal boundary of any state.
    """
    r, w, heads, width = q.shape
    dev = q.device
    lib = _lib.lib()
    ops = [_as_bf16(t, n, dev) for t, n in ((q, "q"), (k, "k"), (v, "v"), (raw_q, "raw_q"), (raw_k, "raw_k"))]
    for t in ops[1:]:
        if t.shape != q.shape:
            raise ValueError("q, k, v, raw_q and raw_k must have the same shape")
    fa = fusion_a if (fusion_a.dtype == _BF16 and fusion_a.is_contiguous() and fusion_a.device == dev) \
        else fusion_a.detach().to(dev, _BF16).contiguous()
    fb = fusion_b if (fusion_b.dtype == _BF16 and fusion_b.is_contiguous() and fusion_b.device == dev) \
        else fusion_b.detach().to(dev, _BF16).contiguous()
    if fa.shape != (heads, width, 3) or fb.shape != (heads, width, 3):
        raise ValueError("fusion_a and fusion_b must have shape [heads, width, 3]")
    feature = states[0].config.fine_writer in FEATURE_WRITERS
    if any((st.config.fine_writer in FEATURE_WRITERS) != feature for st in states):
        raise ValueError("a batch mixes feature-read writers with other fine writers")
    for st in states:
        st._ensure(heads, width, dev, w)
    if (allow_graph and w == 1 and dev.type == "cuda" and _graph_states(states)
            and _BatchGraph.run(states, ops, fa, fb, alpha, out, heads, width)):
        for st in states:
            _bookkeep(st, 1)
        return
    args = _BatchArgs.get(states, w, heads, width, dev)
    for i, st in enumerate(states):
        args.pos[i] = st.position
    stream = torch.cuda.current_stream(dev).cuda_stream
    ws = _Workspace.get(dev, stream, args.nbytes)
    if w == 1:
        _lib.check(lib.tao_decode_step(args.ptrs.data_ptr(), r, args.pos, args.layers, args.cap,
                                       ctypes.byref(args.policy), heads, width,
                                       *(t.data_ptr() for t in ops), fa.data_ptr(), fb.data_ptr(),
                                       float(alpha), out.data_ptr(), ws.data_ptr(), ws.numel(), stream))
    else:
        _lib.check(lib.tao_stream_step(args.ptrs.data_ptr(), r, args.pos, args.cap, ctypes.byref(args.policy),
                                       w, heads, width, *(t.data_ptr() for t in ops), fa.data_ptr(),
                                       fb.data_ptr(), float(alpha), out.data_ptr(), ws.data_ptr(),
                                       ws.numel(), stream))
    for st in states:
        if st.config.fine_writer != "softmax":
            end = st.position + w
            if end - window_start(end - 1) == WINDOW:   # this chunk sealed a block
                st._seal_writer(sealed_at(end - 1))
        _bookkeep(st, w)


def _graph_states(states):
    return all(st.config.q1_history_region_graph and st.config.fine_writer == "softmax" for st in states)


class _HostStage:
    """Device staging of decode operands that arrive in page-locked host memory:
    one [6, R, 1, H, D] bf16 buffer (q, k, v, raw_q, raw_k, output) per (device,
    stream, shape), reused by every call with that shape."""

    cache = {}

    @classmethod
    def get(cls, device, stream, shape):
        key = (device, stream, tuple(shape))
        buf = cls.cache.get(key)
        if buf is None:
            if len(cls.cache) >= 64:
                cls.cache.clear()
            buf = cls.cache[key] = torch.empty((6,) + tuple(shape), dtype=_BF16, device=device)
        return buf


def run_batch_host(states, host_ops, fusion_a, fusion_b, alpha, host_out):
    """One decode token for every state with the operands in page-locked host memory
    and the result written to page-locked host memory.  The SMs move the bytes over
    the host link (one launch in, one out); with graph-configured states the copies
    and the decode step are captured together and a step is one graph launch.  The
    host output is valid once the current stream has reached the step."""
    from .host_io import copy_to_device_many, copy_to_host
    r, w, heads, width = host_ops[0].shape
    if w != 1:
        raise ValueError("host operands are taken one decode token at a time")
    for t in tuple(host_ops) + (host_out,):
        if t.device.type != "cpu" or not t.is_pinned() or t.dtype != _BF16 or not t.is_contiguous():
            raise ValueError("host operands and output must be contiguous page-locked bf16 tensors")
        if t.shape != host_ops[0].shape:
            raise ValueError("q, k, v, raw_q, raw_k and out must have the same shape")
    devs = {st.device for st in states if st.device is not None}
    if len(devs) > 1:
        raise ValueError("a batch spans one device")
    dev = devs.pop() if devs else torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream(dev).cuda_stream
    stage = _HostStage.get(dev, stream, host_ops[0].shape)
    ops, out = [stage[i] for i in range(5)], stage[5]
    if _graph_states(states):
        fa = fusion_a if (fusion_a.dtype == _BF16 and fusion_a.is_contiguous() and fusion_a.device == dev) \
            else fusion_a.detach().to(dev, _BF16).contiguous()
        fb = fusion_b if (fusion_b.dtype == _BF16 and fusion_b.is_contiguous() and fusion_b.device == dev) \
            else fusion_b.detach().to(dev, _BF16).contiguous()
        if fa.shape != (heads, width, 3) or fb.shape != (heads, width, 3):
            raise ValueError("fusion_a and fusion_b must have shape [heads, width, 3]")
        for st in states:
            st._ensure(heads, width, dev, 1)
        if _BatchGraph.run(states, ops, fa, fb, alpha, out, heads, width, host=(host_ops, host_out)):
            for st in states:
                _bookkeep(st, 1)
            return host_out
    copy_to_device_many(ops, list(host_ops))
    run_batch(states, *ops, fusion_a, fusion_b, alpha, out, allow_graph=False)
    copy_to_host(host_out, out)
    return host_out


def _bookkeep_decode(st):
    """``_bookkeep(st, 1)`` for the softmax writer, with the local-length peak settled
    once the window is full (the per-token path of a serving loop)."""
    c = st._counters
    if st.position >= WINDOW:
        c["fusion_pointwise_calls"] += 1
        c["fused_fine_calls"] += 1
        st.position += 1
        if c["peak_local_tokens"] < WINDOW:
            local = st.position - window_start(st.position - 1)
            if local > c["peak_local_tokens"]:
                c["peak_local_tokens"] = local
    else:
        _bookkeep(st, 1)


def _bookkeep(st, w):
    """Host-side cursor and counters after a chunk of ``w`` tokens."""
    c = st._counters
    if st.position >= WINDOW:
        c["fusion_pointwise_calls"] += 1
        if st.config.fine_writer not in FEATURE_WRITERS:   # the feature read is not the fused fine path
            c["fused_fine_calls"] += 1
    else:
        c["fusion_no_history_local_returns"] += 1
    st.position += w
    local = st.position - window_start(st.position - 1)
    if local > c["peak_local_tokens"]:
        c["peak_local_tokens"] = local


class _DecodeGraph:
    """The whole decode step of one state as a CUDA graph over fixed buffers.

    Used when ``config.q1_history_region_graph`` is set (reference
    ``HistoryRegionGraph``, history_region_graph.py:10-113, which captures the
    history read only and re-captures after every seal).  Here the graph holds the
    route, fused decode and seal kernels of ``tao_decode_step`` in graph mode: the
    route and seal kernels read the cursor from the device state and return early
    on tokens that neither refresh nor seal, so a seal needs no re-capture.  The
    graph is captured again only when the fine bank grows (new grid sizes and
    buffers), or when alpha or the operand shape changes.
    """

    def __init__(self, st, heads, width, alpha):
        dev = st.device
        lib = _lib.lib()
        self.key = (st.cap_fines, st._desc.data_ptr(), heads, width, float(alpha), _policy_key(st.config))
        self.inp = torch.zeros(5, 1, 1, heads, width, dtype=_BF16, device=dev)   # q, k, v, raw_q, raw_k
        self.fab = torch.zeros(2, heads, width, 3, dtype=_BF16, device=dev)      # fusion_a, fusion_b
        self.out = torch.zeros(1, 1, heads, width, dtype=_BF16, device=dev)
        self.ptrs = torch.tensor([st._desc.data_ptr()], dtype=torch.int64, device=dev)
        self.policy = policy_for(st.config)
        self.pos = (ctypes.c_int64 * 1)(st.position)
        self.cap = (ctypes.c_int32 * 1)(st.cap_fines)
        self.layer = (ctypes.c_int32 * 1)(st.layer_index)
        nbytes = lib.tao_stream_workspace_bytes(1, 1, heads, width, ROUTE_CAP, ctypes.byref(self.policy))
        self.ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        _graph_workspaces(dev).add(self.ws)
        self.graph = torch.cuda.CUDAGraph()
        rc = 0
        lib.tao_decode_graph_mode(1)
        try:
            # "relaxed": the launcher may set kernel shared-memory attributes during capture
            with torch.cuda.graph(self.graph, capture_error_mode="relaxed"):
                rc = lib.tao_decode_step(self.ptrs.data_ptr(), 1, self.pos, self.layer, self.cap,
                                         ctypes.byref(self.policy), heads, width,
                                         *(self.inp[i].data_ptr() for i in range(5)),
                                         self.fab[0].data_ptr(), self.fab[1].data_ptr(), float(alpha),
                                         self.out.data_ptr(), self.ws.data_ptr(), self.ws.numel(),
                                         torch.cuda.current_stream(dev).cuda_stream)
        finally:
            lib.tao_decode_graph_mode(0)
        _lib.check(rc)

    @staticmethod
    def step(st, q, k, v, raw_q, raw_k, fusion_a, fusion_b, alpha, out):
        r, w, heads, width = q.shape
        if r != 1 or w != 1:
            raise ValueError("graph decode takes [1, 1, heads, width] operands")
        dev = q.device
        ops = [_as_bf16(t, n, dev) for t, n in ((q, "q"), (k, "k"), (v, "v"), (raw_q, "raw_q"), (raw_k, "raw_k"))]
        for t in ops[1:]:
            if t.shape != q.shape:
                raise ValueError("q, k, v, raw_q and raw_k must have the same shape")
        if fusion_a.shape != (heads, width, 3) or fusion_b.shape != (heads, width, 3):
            raise ValueError("fusion_a and fusion_b must have shape [heads, width, 3]")
        st._ensure(heads, width, dev, 1)   # may grow the fine bank (new buffers)
        g = st._graph
        key = (st.cap_fines, st._desc.data_ptr(), heads, width, float(alpha), _policy_key(st.config))
        if g is None or g.key != key:
            g = st._graph = _DecodeGraph(st, heads, width, alpha)
        for i, t in enumerate(ops):
            g.inp[i].copy_(t)
        g.fab[0].copy_(fusion_a)
        g.fab[1].copy_(fusion_b)
        g.graph.replay()
        out.copy_(g.out)
        _bookkeep(st, 1)


# Workspaces of live captured graphs, per device (weak: a graph that is replaced
# or evicted frees its workspace and drops out of the error check).
_GRAPH_WORKSPACES = {}


def _graph_workspaces(device):
    return _GRAPH_WORKSPACES.setdefault(device, weakref.WeakSet())


class _BatchGraph:
    """Graph mode for ``tao_attention_decode_batch`` (states configured with
    ``q1_history_region_graph``): the decode step of the whole batch, captured over
    the caller's own operand buffers.  A step is captured the second time the same
    states, capacities, alpha and operand addresses are seen in a row (callers that
    reuse their buffers, as graph users do) and replayed from then on; other calls
    run eagerly.  Like ``_DecodeGraph``, nothing is re-captured at a seal."""

    cache = {}      # key -> _BatchGraph
    last = None     # key of the previous eager call

    def __init__(self, states, ops, fa, fb, alpha, out, heads, width, host=None):
        dev = ops[0].device
        lib = _lib.lib()
        r = len(states)
        if host is not None:   # page-locked host operands and output: copies captured with the step
            host_ops, host_out = host
            n = len(ops)
            self.copy_dst = (ctypes.c_void_p * n)(*[t.data_ptr() for t in ops])
            self.copy_src = (ctypes.c_void_p * n)(*[t.data_ptr() for t in host_ops])
            self.copy_bytes = (ctypes.c_size_t * n)(*[t.numel() * t.element_size() for t in host_ops])
            self.host_out = host_out
        self.host = host is not None
        self.ptrs = torch.tensor([st._desc.data_ptr() for st in states], dtype=torch.int64, device=dev)
        self.policy = policy_for(states[0].config)
        self.pos = (ctypes.c_int64 * r)(*[st.position for st in states])
        self.cap = (ctypes.c_int32 * r)(*[st.cap_fines for st in states])
        self.layers = (ctypes.c_int32 * r)(*[st.layer_index for st in states])
        nbytes = lib.tao_stream_workspace_bytes(r, 1, heads, width, ROUTE_CAP, ctypes.byref(self.policy))
        self.ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        _graph_workspaces(dev).add(self.ws)
        self.graph = torch.cuda.CUDAGraph()
        rc = 0
        lib.tao_decode_graph_mode(1)
        try:
            with torch.cuda.graph(self.graph, capture_error_mode="relaxed"):
                stream = torch.cuda.current_stream(dev).cuda_stream
                if self.host:
                    rc = lib.tao_copy_host_to_device_many(self.copy_dst, self.copy_src, self.copy_bytes,
                                                          len(ops), stream)
                if rc == 0:
                    rc = lib.tao_decode_step(self.ptrs.data_ptr(), r, self.pos, self.layers, self.cap,
                                             ctypes.byref(self.policy), heads, width,
                                             *(t.data_ptr() for t in ops), fa.data_ptr(), fb.data_ptr(),
                                             float(alpha), out.data_ptr(), self.ws.data_ptr(), self.ws.numel(),
                                             stream)
                if rc == 0 and self.host:
                    rc = lib.tao_copy_device_to_host(self.host_out.data_ptr(), out.data_ptr(),
                                                     out.numel() * out.element_size(), stream)
        finally:
            lib.tao_decode_graph_mode(0)
        _lib.check(rc)

    @classmethod
    def run(cls, states, ops, fa, fb, alpha, out, heads, width, host=None):
        """Replay (or capture and replay) the batch step; False = run it eagerly.
        ``host`` = (host operands, host output) when the step's operands arrive in,
        and its result goes back to, page-locked host memory."""
        key = (tuple((st._desc.data_ptr(), st.cap_fines, st.layer_index) for st in states), heads, width,
               float(alpha), tuple(t.data_ptr() for t in ops), fa.data_ptr(), fb.data_ptr(), out.data_ptr(),
               _policy_key(states[0].config),
               None if host is None else (tuple(t.data_ptr() for t in host[0]), host[1].data_ptr()))
        g = cls.cache.get(key)
        if g is None:
            if cls.last != key:
                cls.last = key
                return False
            if len(cls.cache) >= 8:
                cls.cache.clear()
            g = cls.cache[key] = cls(states, ops, fa, fb, alpha, out, heads, width, host)
        g.graph.replay()
        return True


def check_device(device=None):
    """Raise if a kernel on ``device`` reported an error since the last check."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    current = torch.cuda.current_stream(dev).cuda_stream
    flags = ctypes.c_int(0)
    total = 0
    # the words of every stream's workspace are read on the current stream after a
    # device-wide synchronisation (another stream's handle may be gone by now)
    torch.cuda.synchronize(dev)
    for ws in [buf for _, buf in _Workspace.on_device(dev)] + list(_GRAPH_WORKSPACES.get(dev, ())):
        _lib.check(_lib.lib().tao_stream_check(ws.data_ptr(), ctypes.byref(flags), current))
        total |= flags.value
    return total


def route_count_at(pos, layer, config):
    """Selected fines M held by a state serving ``pos`` (from its latest refresh)."""
    if pos < WINDOW:
        return 0
    first_turn = WINDOW + config.layer_stagger * layer
    if pos < first_turn:
        last = WINDOW
    else:
        last = first_turn + ((pos - first_turn) // config.route_period) * config.route_period
    s = sealed_at(last)
    return routed_counts(s // GROUP, s % GROUP, config)[2]


def decode_bytes(states):
    """Algorithmic HBM bytes of one decode step's main phase for these states:
    local K and V of every key in the window (current token included), the
    selected fine matrices with their z / page z / page weight rows, q and raw_q."""
    total = 0
    for st in states:
        h, d, pos = st.heads, st.width, st.position
        keys = pos - window_start(pos) + 1
        m = route_count_at(pos, st.layer_index, st.config)
        total += keys * h * d * 2 * 2 + m * h * (d * d * 2 + 3 * d * 2) + 2 * h * d * 2
    return total


class BatchDecoder:
    """Low-overhead decode loop over the C ABI for a fixed set of states.

    ``step(q, k, v, raw_q, raw_k, out)`` takes device pointers of
    [len(states), 1, H, D] bf16 buffers and advances every state by one token.
    Capacity is reserved up front with ``reserve(tokens)``; the loop performs no
    allocation and no synchronisation.
    """

    def __init__(self, states, fusion_a, fusion_b, alpha, device):
        self.states = list(states)
        self.dev = torch.device(device)
        st0 = self.states[0]
        self.heads, self.width = st0.heads, st0.width
        self.fa = fusion_a.detach().to(self.dev, _BF16).contiguous()
        self.fb = fusion_b.detach().to(self.dev, _BF16).contiguous()
        self.alpha = float(alpha)
        self.policy = policy_for(st0.config)
        self.lib = _lib.lib()
        self.r = len(self.states)
        self.pos = (ctypes.c_int64 * self.r)()
        self.cap = (ctypes.c_int32 * self.r)()
        self.layers = (ctypes.c_int32 * self.r)(*[st.layer_index for st in self.states])
        nbytes = self.lib.tao_stream_workspace_bytes(self.r, 1, self.heads, self.width, ROUTE_CAP,
                                                     ctypes.byref(self.policy))
        self.ws = torch.zeros(nbytes, dtype=torch.uint8, device=self.dev)
        self._sync_ptrs()

    def _sync_ptrs(self):
        self.ptrs = torch.tensor([st._desc.data_ptr() for st in self.states], dtype=torch.int64,
                                 device=self.dev)
        for i, st in enumerate(self.states):
            self.pos[i] = st.position
            self.cap[i] = st.cap_fines

    def reserve(self, tokens):
        """Make every state's fine bank hold ``tokens`` more tokens of history."""
        for st in self.states:
            need = sealed_at(st.position + tokens) + 1
            if need > st.cap_fines:
                st._grow(need)
        self._sync_ptrs()

    def step(self, q, k, v, raw_q, raw_k, out, stream=None):
        s = torch.cuda.current_stream(self.dev).cuda_stream if stream is None else stream
        _lib.check(self.lib.tao_decode_step(
            self.ptrs.data_ptr(), self.r, self.pos, self.layers, self.cap, ctypes.byref(self.policy),
            self.heads, self.width, q, k, v, raw_q, raw_k, self.fa.data_ptr(), self.fb.data_ptr(),
            self.alpha, out, self.ws.data_ptr(), self.ws.numel(), s))
        for i, st in enumerate(self.states):
            st.position += 1
            self.pos[i] = st.position

    def check(self):
        flags = ctypes.c_int(0)
        _lib.check(self.lib.tao_stream_check(self.ws.data_ptr(), ctypes.byref(flags),
                                             torch.cuda.current_stream(self.dev).cuda_stream))


class DecodeSession:
    """A fixed batch of requests decoded one token per step, operands and results
    in page-locked host memory: the serving loop of one layer for callers whose
    tokens arrive in, and leave through, host memory.

    ``inputs``: page-locked [5, R, 1, H, D] bf16 (q, k, v, raw_q, raw_k of the next
    token of every request), filled by the caller before each ``step()``;
    ``output``: page-locked [R, 1, H, D] bf16, valid after ``wait()``.  ``step()``
    launches the decode step through ``tao_decode_step_host``: its routing launch
    brings the operands in over the host link and the fused kernel writes the output
    rows, then a completion word, into page-locked memory; with states configured
    for graphs (``q1_history_region_graph``) the step is captured once and a step is
    one graph launch, and ``wait()`` spins on the completion word.  ``reserve`` tokens of fine-bank capacity are allocated up
    front, so the loop allocates nothing and the graph is not captured again within
    them.  The states advance exactly as with ``tao_attention_decode_batch``; while a
    session runs they advance only through it (a caller that advances one otherwise
    calls ``reserve`` before the next ``step``, which re-derives when the banks grow).
    """

    def __init__(self, states, fusion_a, fusion_b, alpha, reserve=4096):
        self.states = list(states)
        if not self.states or len({id(s) for s in self.states}) != len(self.states):
            raise ValueError("a session takes distinct states")
        devs = {st.device for st in self.states}
        if None in devs or len(devs) != 1:
            raise ValueError("the states of a session must be allocated on one device (prefill them first)")
        self.dev = devs.pop()
        st0 = self.states[0]
        self.heads, self.width = st0.heads, st0.width
        if any((st.heads, st.width) != (self.heads, self.width) for st in self.states):
            raise ValueError("the states of a session share one head count and width")
        if any(_policy_key(st.config) != _policy_key(st0.config) for st in self.states):
            raise ValueError("the states of a session share one routing policy")
        if st0.config.fine_writer != "softmax":
            raise ValueError("sessions serve the softmax fine writer")
        self.r = len(self.states)
        self.graph_mode = _graph_states(self.states)
        self.lib = _lib.lib()
        self.stream = torch.cuda.current_stream(self.dev)
        with torch.cuda.device(self.dev):
            self.fa = fusion_a.detach().to(self.dev, _BF16).contiguous()
            self.fb = fusion_b.detach().to(self.dev, _BF16).contiguous()
            if self.fa.shape != (self.heads, self.width, 3) or self.fb.shape != self.fa.shape:
                raise ValueError("fusion_a and fusion_b must have shape [heads, width, 3]")
            self.alpha = float(alpha)
            shape = (self.r, 1, self.heads, self.width)
            self.inputs = torch.zeros((5,) + shape, dtype=_BF16).pin_memory()
            self.output = torch.zeros(shape, dtype=_BF16).pin_memory()
            self.stage = torch.zeros((5,) + shape, dtype=_BF16, device=self.dev)
            self.done = torch.zeros(1, dtype=torch.int32).pin_memory()   # completion word
            self._done_ptr = ctypes.c_void_p(self.done.data_ptr())
            self.seq = 0                                                 # steps launched
            self._stream_ptr = ctypes.c_void_p(self.stream.cuda_stream)
            self.policy = policy_for(st0.config)
            self.layers = (ctypes.c_int32 * self.r)(*[st.layer_index for st in self.states])
            self.pos = (ctypes.c_int64 * self.r)()
            self.cap = (ctypes.c_int32 * self.r)()
            nbytes = self.lib.tao_stream_workspace_bytes(self.r, 1, self.heads, self.width, ROUTE_CAP,
                                                         ctypes.byref(self.policy))
            self.ws = torch.zeros(nbytes, dtype=torch.uint8, device=self.dev)
            _graph_workspaces(self.dev).add(self.ws)
            self.graph = None
            self.reserve(reserve)

    def reserve(self, tokens):
        """Fine-bank capacity for ``tokens`` more tokens of every request (may grow
        the banks; a captured step is then captured again at the next step)."""
        grew = False
        for st in self.states:
            need = sealed_at(st.position + tokens) + 1
            if need > st.cap_fines:
                st._grow(need)
                grew = True
        self.ptrs = torch.tensor([st._desc.data_ptr() for st in self.states], dtype=torch.int64,
                                 device=self.dev)
        for i, st in enumerate(self.states):
            self.cap[i] = st.cap_fines
        if grew:
            self.graph = None
        # steps until some state's next seal would exceed its fine-bank capacity
        # (sealed_at(p + 1) + 1 > cap from p = 767 + 256 (cap - 1) on)
        self._steps_left = min(767 + FINE * (st.cap_fines - 1) - st.position for st in self.states)

    def _launch(self, stream):
        # one routing launch that also brings the operands in over the host link, the
        # fused kernel writing the outputs straight into the page-locked output and
        # then the step's sequence number into the completion word
        return self.lib.tao_decode_step_host(self.ptrs.data_ptr(), self.r, self.pos, self.layers, self.cap,
                                             ctypes.byref(self.policy), self.heads, self.width,
                                             self.inputs.data_ptr(), self.stage.data_ptr(),
                                             self.output.data_ptr(), self.done.data_ptr(), self.fa.data_ptr(),
                                             self.fb.data_ptr(), self.alpha, self.ws.data_ptr(), self.ws.numel(),
                                             stream)

    def _capture(self):
        self.graph = torch.cuda.CUDAGraph()
        rc = 0
        self.lib.tao_decode_graph_mode(1)
        try:
            with torch.cuda.graph(self.graph, capture_error_mode="relaxed"):
                rc = self._launch(torch.cuda.current_stream(self.dev).cuda_stream)
        finally:
            self.lib.tao_decode_graph_mode(0)
        _lib.check(rc)
        self._exec = ctypes.c_void_p(self.graph.raw_cuda_graph_exec())

    def step(self):
        """Decode the token in ``inputs`` for every request (asynchronous)."""
        if self._steps_left <= 0:
            self.reserve(4096)
        if self.graph_mode:
            if self.graph is None:
                self._sync_positions()
                with torch.cuda.stream(self.stream):
                    self._capture()
            _lib.check(self.lib.tao_graph_launch(self._exec, self._stream_ptr))
        else:
            self._sync_positions()
            _lib.check(self._launch(self._stream_ptr))
        self._steps_left -= 1
        self.seq += 1
        for st in self.states:
            _bookkeep_decode(st)

    def _sync_positions(self):
        # the host cursors the C ABI validates (a captured step decides on the device)
        for i, st in enumerate(self.states):
            self.pos[i] = st.position

    def wait(self):
        """Block until the last step's ``output`` is in host memory.

        The host thread spins on the completion word the fused kernel writes after the
        step's last output row; the step's seal kernel (when a window fills) may still
        be running, in order on the session's stream, when this returns.  On a device
        error (no completion) the stream is synchronised and the error raised."""
        if self.lib.tao_host_wait(self._done_ptr, self.seq, 5_000_000) != 0:
            self.stream.synchronize()
            self.check()
            _lib.check(self.lib.tao_host_wait(self._done_ptr, self.seq, 0))
        return self.output

    def check(self):
        """Raise if a kernel of this session reported an error."""
        flags = ctypes.c_int(0)
        _lib.check(self.lib.tao_stream_check(self.ws.data_ptr(), ctypes.byref(flags), self.stream.cuda_stream))
