"""CPU oracle for the TaoMemory attention operator -- TEST INFRASTRUCTURE ONLY.

This module restates the reference algorithm (LaurenceLong/tao-memory,
``tao_attention/``) with plain PyTorch CPU tensor operations, keeping every
bf16 rounding point of the reference.  Only ``tests/``, ``__graft_entry__.smoke()``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it,
and only as the checker or the timed CPU baseline.  The product package
``tao_memory_b200`` never imports it and has no CPU fallback.

Pinning: ``tests/golden/*.pt`` hold outputs of the unmodified reference run in a
container where it was importable (script: ``tests/golden/make_golden.py``);
``tests/test_oracle_golden.py`` checks this restatement against them.

Scope: the preset path ``index_only_page_memo`` (``coarse_index_only=True``,
``fine_writer="softmax"``), streaming prefill/decode for one request and
training forward/backward for batch B; for streaming also
``fine_writer="regularized_association"``, ``"feature_mass_association"`` and
``"structured_gram_association"`` on the same preset.

Rounding conventions (probed against torch CPU 2.11):
* ``F.softmax``, ``Tensor.sum`` and ``Tensor.exp`` on bf16 compute in fp32 and
  round once;
* ``torch.logsumexp`` on bf16 is a composite (amax, sub, exp, sum, log, add)
  that rounds to bf16 after every step.
"""

import math

import torch
import torch.nn.functional as F

BF16 = torch.bfloat16
F32 = torch.float32


def _r(x):
    """Round an fp32 tensor to bf16 and back (a reference ``.to(bf16)`` point)."""
    return x.to(BF16).to(F32)


# --------------------------------------------------------------------------
# Integer schedule (tao_stream.py:29-53, config.py:54-60)
# --------------------------------------------------------------------------

def budget(count, root_scale=2, offset=2):
    if count <= 0:
        return 0
    square = root_scale * count
    root = math.isqrt(square)
    root += int(root * root < square)
    return min(count, root + offset)


def routed_counts(completed, pending, group=8, root_scale=2, offset=2):
    """tao_stream.py:29-37."""
    coarse_budget = budget(group * completed, root_scale, offset)
    coarse = min(completed, (2 * coarse_budget + group - 1) // group)
    eligible = group * coarse + pending
    return coarse, eligible, min(eligible, budget(group * completed + pending,
                                                  root_scale, offset))


def topk_oldest(scores, count):
    """Stable descending argsort; the lower (older) index wins exact ties
    (tao_stream.py:50-53)."""
    return scores.argsort(dim=-1, descending=True, stable=True)[
        ..., :min(count, scores.shape[-1])]


# --------------------------------------------------------------------------
# Kernels restated (Triton -> torch CPU)
# --------------------------------------------------------------------------

def local_attention(q, k, v):
    """Suffix-aligned causal SDPA on [B,T,H,D] (flash_attention.py:16-37)."""
    query, key, value = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    if q.shape[1] == k.shape[1]:
        out = F.scaled_dot_product_attention(query, key, value, is_causal=True)
    elif q.shape[1] == 1:
        out = F.scaled_dot_product_attention(query, key, value, is_causal=False)
    else:
        rows = k.shape[1] - q.shape[1] + torch.arange(q.shape[1])
        cols = torch.arange(k.shape[1])
        allowed = cols[None, :] <= rows[:, None]
        out = F.scaled_dot_product_attention(query, key, value, attn_mask=allowed,
                                             is_causal=False)
    return out.transpose(1, 2)


def seal_block(raw_k, v):
    """Softmax fine writer for one block [B,256,H,D] -> z [B,H,D], C [B,H,D,D]
    (tao_stream.py:66-76)."""
    dt = raw_k.dtype
    maximum = raw_k.amax(dim=1, keepdim=True)
    exponent = (raw_k - maximum).exp().to(dt)
    partition = exponent.sum(dim=1, keepdim=True).to(dt)
    prob = (exponent / partition).to(dt)
    z = (maximum.squeeze(1) + partition.squeeze(1).log()).to(dt)
    with torch.autocast(device_type="cpu", enabled=False):
        c = torch.einsum("bthd,bthe->bhde", prob, v).to(dt)
    return z, c


def association_statistics(raw_k, v, with_mass=False):
    """Association-writer statistics of one block [B,256,H,D] (association_writer.py:11-18):
    u = bf16(fp32 softmax over channels), G = u^T u and X = u^T v in fp32, [B,H,D,D];
    with_mass adds the fp32 feature mass sum_t u [B,H,D]."""
    with torch.autocast(device_type="cpu", enabled=False):
        u = raw_k.float().softmax(dim=-1).to(BF16).transpose(1, 2).float()
        values = v.transpose(1, 2).float()
        gram, cross = u.transpose(-1, -2) @ u, u.transpose(-1, -2) @ values
        return (gram, cross, u.sum(dim=-2)) if with_mass else (gram, cross)


def association_matrix(gram, cross, unchecked=False):
    """Regularised solve (association_writer.py:21-32): C = bf16(A^{-1} X) with
    A = G + (trace(G)/D) I through a Cholesky factor (unchecked: no error raised
    for a failed factorisation, as the feature-mass writer asks)."""
    with torch.autocast(device_type="cpu", enabled=False):
        width = gram.shape[-1]
        reg = gram.diagonal(dim1=-2, dim2=-1).sum(-1) / width
        system = gram + reg[..., None, None] * torch.eye(width, dtype=F32)
        if unchecked:
            factor, _ = torch.linalg.cholesky_ex(system, upper=False, check_errors=False)
        else:
            factor = torch.linalg.cholesky(system)
        return torch.cholesky_solve(cross, factor).to(BF16)


FEATURE_WRITERS = ("feature_mass_association", "structured_gram_association")


def structured_statistics(raw_k, v):
    """Structured-Gram writer statistics (structured_writer.py:5-14), no dense Gram:
    with u as in association_statistics, the fp32 square mass sum_t u*u and mass
    sum_t u per channel [B,H,D] and X = u^T v [B,H,D,D].  Returns (square, X, mass)."""
    with torch.autocast(device_type="cpu", enabled=False):
        u = raw_k.float().softmax(dim=-1).to(BF16).transpose(1, 2).float()
        values = v.transpose(1, 2).float()
        return (u * u).sum(-2), u.transpose(-1, -2) @ values, u.sum(-2)


def structured_matrix(square, cross, mass, count):
    """Closed-form structured inverse applied to X (structured_writer.py:17-34), fp32
    throughout, C = bf16 at the end.  The Gram is modelled per channel as the
    clamped variance var = square - mass^2/count plus a ridge (mean square mass)
    on the diagonal, a rank-one term along t = var/diag (dropped when every var is
    zero) and the rank-one mass term, removed by Sherman-Morrison with denominator
    count + mass . hm.  The fp32 operations run in the reference's order."""
    with torch.autocast(device_type="cpu", enabled=False):
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
        return (hx - hm.unsqueeze(-1) * mhx.unsqueeze(-2) / den.unsqueeze(-1)).to(BF16)


def feature_read(h, selected_z, selected_id, fine_c):
    """Feature-mass read (association_writer.py:43-53, indirect_fine.py:13-33):
    mass_m = sum_d h_d exp(z_m,d) in fp32, channel_m = bf16(h * mass_m / sum_m mass),
    fine = bf16(sum_m sum_d channel_m,d C_m[d, :]) accumulated in fp32, no denominator.
    h [B,Q,H,D] bf16, selected_z [B,Q,H,M,D], selected_id [B,Q,H,M], fine_c [B,H,S,D,D]."""
    with torch.autocast(device_type="cpu", enabled=False):
        query = h.float().unsqueeze(-2)
        mass = (query * selected_z.float().exp()).sum(-1)
        mixture = mass / mass.sum(-1, keepdim=True)
        channel = (mixture.unsqueeze(-1) * query).to(h.dtype)
        return _SelectedContraction.apply(channel, selected_id, fine_c)


class _SelectedContraction(torch.autograd.Function):
    """selected_fine_numerator / _SelectedContraction (indirect_fine.py:65-133)
    restated: out = bf16(sum_m channel_m . C_m) in fp32; the adjoints with the
    reference's rounding points: d channel = bf16(g . C^T) per selected pair and
    dC = bf16(fp32 sum over the pairs that selected the fine of channel^T g)."""

    @staticmethod
    def forward(ctx, channel, ids, fine_c):
        b, q, h, m = ids.shape
        bi = torch.arange(b)[:, None, None, None]
        hi = torch.arange(h)[None, None, :, None]
        csel = fine_c[bi, hi, ids].float()
        ctx.save_for_backward(channel, ids, fine_c)
        return torch.einsum("bqhmd,bqhmde->bqhe", channel.float(), csel).to(channel.dtype)

    @staticmethod
    def backward(ctx, g):
        channel, ids, fine_c = ctx.saved_tensors
        b, q, h, m = ids.shape
        bi = torch.arange(b)[:, None, None, None]
        hi = torch.arange(h)[None, None, :, None]
        csel = fine_c[bi, hi, ids].float()
        gf = g.float()
        d_channel = torch.einsum("bqhe,bqhmde->bqhmd", gf, csel).to(channel.dtype)
        outer = torch.einsum("bqhmd,bqhe->bqhmde", channel.float(), gf)
        dc = torch.zeros(fine_c.shape, dtype=F32)
        dc.index_put_((bi.expand(b, q, h, m), hi.expand(b, q, h, m), ids), outer, accumulate=True)
        return d_channel, None, dc.to(fine_c.dtype)


def seal_all(raw_k, v, fine=256, writer="softmax"):
    """Training writer over all complete blocks but the last (tao_stream.py:80-123):
    returns z [B,H,S,D], C [B,H,S,D,D] with S = T//fine - 1.  With
    writer="regularized_association" z stays the softmax writer's and C is the
    regularised association matrix of each block (tao_stream.py:113-117)."""
    b, total, heads, d = raw_k.shape
    s = total // fine - 1
    keys = raw_k[:, :s * fine].reshape(b, s, fine, heads, d)
    values = v[:, :s * fine].reshape(b, s, fine, heads, d)
    dt = raw_k.dtype
    maximum = keys.amax(dim=2, keepdim=True)
    exponent = (keys - maximum).exp().to(dt)
    partition = exponent.sum(dim=2, keepdim=True).to(dt)
    prob = (exponent / partition).to(dt)
    z = (maximum.squeeze(2) + partition.squeeze(2).log()).to(dt)
    if writer == "regularized_association":
        gram, cross = association_statistics(keys.reshape(b * s, fine, heads, d),
                                             values.reshape(b * s, fine, heads, d))
        c = association_matrix(gram, cross).reshape(b, s, heads, d, d).permute(0, 2, 1, 3, 4)
        return z.permute(0, 2, 1, 3), c
    with torch.autocast(device_type="cpu", enabled=False):
        c = torch.einsum("bsihd,bsihe->bhsde", prob, values).to(dt)
    return z.permute(0, 2, 1, 3), c


def seal_all_feature(raw_k, v, writer, fine=256):
    """Training writer of the feature-read writers over all complete blocks but the
    last (_seal_training_all, tao_stream.py:87-106): z = bf16(log mass) per block and
    C from the unchecked regularised solve (feature-mass) or the structured inverse
    (structured-Gram, count = 256).  Returns z [B,H,S,D], C [B,H,S,D,D] and the fp32
    feature mass [B,H,S,D] that the page log-masses are built from."""
    b, total, heads, d = raw_k.shape
    s = total // fine - 1
    keys = raw_k[:, :s * fine].reshape(b * s, fine, heads, d)
    values = v[:, :s * fine].reshape(b * s, fine, heads, d)
    if writer == "structured_gram_association":
        square, cross, mass = structured_statistics(keys, values)
        c = structured_matrix(square, cross, mass, fine)
    else:
        gram, cross, mass = association_statistics(keys, values, with_mass=True)
        c = association_matrix(gram, cross, unchecked=True)
    c = c.reshape(b, s, heads, d, d).permute(0, 2, 1, 3, 4)
    mass = mass.reshape(b, s, heads, d).permute(0, 2, 1, 3)
    return mass.log().to(raw_k.dtype), c, mass


def chronological_sum(x, dim):
    """Sum along ``dim`` one element after another in index order (fp32), the order of
    chronological_sum (association_writer.py:35-40)."""
    total = x.select(dim, 0)
    for i in range(1, x.shape[dim]):
        total = total + x.select(dim, i)
    return total


def fine_read(hv, page_z, fine_z, selected_id, fine_c, group=8):
    """query_fresh_fine.py:30-69 restated.

    hv [B,Q,H,P,D], page_z [B,H,P,D], fine_z [B,H,S,D], selected_id [B,Q,H,M],
    fine_c [B,H,S,D,D] -> (channel [B,Q,H,M,D], num, den, fine).
    """
    b, q, h, p, d = hv.shape
    m = selected_id.shape[-1]
    ids = selected_id.expand(b, q, h, m)
    page = ids // group
    idx = ids[..., None].expand(b, q, h, m, d)
    z = fine_z[:, None].expand(b, q, h, -1, d).gather(3, idx).float()
    pz = page_z[:, None].expand(b, q, h, -1, d).gather(3, page[..., None].expand(b, q, h, m, d)).float()
    hvs = hv.gather(3, page[..., None].expand(b, q, h, m, d)).float()
    w = _r(torch.exp(_r(z - pz)))
    ch = _r(hvs * w)
    bi = torch.arange(b)[:, None, None, None]
    hi = torch.arange(h)[None, None, :, None]
    csel = fine_c[bi, hi, ids].float()
    acc = torch.einsum("bqhmd,bqhmde->bqhe", ch, csel)
    num = acc.to(hv.dtype)
    chan = ch.to(hv.dtype)
    den = chan.sum(-1).sum(-1, keepdim=True).to(hv.dtype)
    return chan, num, den, (num / den).to(hv.dtype)


def fusion_scores(raw_q, a, b, coarse_present, fine_present):
    """fusion_pointwise.py:10-47 restated -> [B,T,H,D,3] in raw_q.dtype."""
    lb = math.log(int(coarse_present) + int(fine_present)) if (coarse_present or fine_present) else 0.0
    qf = raw_q.float()[..., None]
    s = _r(_r(_r(a.float()) * qf) + _r(b.float()))
    s0 = _r(s[..., 0] + _r(torch.tensor(lb)))
    s1 = s[..., 1] if coarse_present else torch.full_like(s0, -math.inf)
    s2 = s[..., 2] if fine_present else torch.full_like(s0, -math.inf)
    return torch.stack((s0, s1, s2), -1).to(raw_q.dtype)


def fusion_weighted_sum(rho, local, coarse, fine, gain):
    """fusion_pointwise.py:50-92 restated (every cast kept)."""
    g = gain.float()
    rl, rc, rf = (rho[..., i].float() for i in range(3))
    lt = _r(rl * _r(2.0 * local.float()))
    ct = _r(rc * _r(g * coarse.float()))
    ft = _r(rf * _r(g * fine.float()))
    return _r(_r(lt + ct) + ft).to(local.dtype)


def fuse_inference(raw_q, local, fine, fa, fb, alpha, fine_on, coarse=None, coarse_on=False):
    """operator.py:86-99: 3-way pointwise gate; no history -> local."""
    if not (fine_on or coarse_on):
        return local
    score = fusion_scores(raw_q, fa, fb, coarse_on, fine_on)
    rho = F.softmax(score, dim=-1).to(raw_q.dtype)
    gain = torch.full((), 2 * alpha, dtype=raw_q.dtype)
    return fusion_weighted_sum(rho, local, torch.zeros_like(fine) if coarse is None else coarse, fine, gain)


def page_matrix(page_fine_z, page_z, page_fine_c):
    """Coarse page matrix of a completed page (tao_stream.py:486-500, softmax
    writer): w_s = bf16(exp(bf16(z_s - page_z))) per fine s of the page, then
    C_page = bf16(sum_s w_s[d] * C_s[d, e]) (einsum in fp32, one rounding).
    page_fine_z [B,H,8,D], page_z [B,H,D], page_fine_c [B,H,8,D,D] -> [B,H,D,D]."""
    dt = page_fine_z.dtype
    weight = (page_fine_z - page_z.unsqueeze(2)).exp().to(dt)
    with torch.autocast(device_type="cpu", enabled=False):
        return torch.einsum("bhsd,bhsde->bhde", weight, page_fine_c).to(dt)


def coarse_read(h, page_z, page_c):
    """Coarse value read (tao_stream.py:299-305): over the completed pages p,
    coarse = bf16(sum_p sum_d bf16(h[d] * softmax_p(page_z)[p, d]) * C_p[d, e]).
    h [B,T,H,D] (bf16 softmax of raw_q), page_z [B,H,P,D] (completed pages only),
    page_c [B,H,P,D,D]."""
    dt = h.dtype
    weight = F.softmax(page_z, dim=2).to(dt)
    chv = (h.unsqueeze(3) * weight[:, None]).to(dt)
    with torch.autocast(device_type="cpu", enabled=False):
        return torch.einsum("bthpd,bhpde->bthe", chv, page_c).to(dt)


# --------------------------------------------------------------------------
# Streaming state (tao_stream.py:126-527, 790-1094) -- preset path only
# --------------------------------------------------------------------------

class OracleStream:
    """One request's one-layer state: exact local window + sealed fines + pages."""

    FINE, KEEP, GROUP, PERIOD, STAGGER = 256, 512, 8, 24, 2

    def __init__(self, layer_index=0, fine_writer="softmax", coarse_index_only=True):
        self.layer_index = layer_index
        self.fine_writer = fine_writer
        self.coarse_index_only = coarse_index_only
        self.page_c = []               # [1,H,D,D] per completed page (coarse value branch only)
        self.coarse_parts, self.last_coarse = [], None
        self.pending_gram = self.pending_cross = None   # fp32 writer statistics (association writers)
        self.pending_mass = None                        # fp32 feature mass (feature-mass writers)
        self.pending_square_mass = None                 # fp32 sum u*u (structured-Gram writer)
        self.position = 0
        self.local = None              # (k, v, raw_k) [1,L,H,D]
        self.pages = []                # (page_z [1,H,D], fine_z [1,H,8,D])
        self.pending = []              # fine_z [1,H,D]
        self.fine_c = None             # [1,H,S,D,D]
        self.route_ids = None          # (chosen_page [1,1,H,K], selected_id [1,1,H,M]) int64
        self.state_version = 0
        self.route_refreshes = 0
        self.fine_seal_events = 0

    @property
    def serve_limit(self):
        return self.KEEP + self.FINE

    def next_chunk(self, desired):
        current = 0 if self.local is None else self.local[0].shape[1]
        return min(desired, self.FINE, self.serve_limit - current)

    # -- history ---------------------------------------------------------
    def _page_tables(self, dtype):
        page_z = [pz for pz, _ in self.pages]
        fine_z = [fz for _, fz in self.pages]
        if self.pending:
            pending_z = torch.stack(self.pending, dim=2)
            page_z.append(self.pending_mass.log().to(dtype) if self.fine_writer in FEATURE_WRITERS
                          else torch.logsumexp(pending_z, dim=2).to(dtype))
            fine_z.append(pending_z)
        page_z = torch.stack(page_z, dim=2)
        return page_z, torch.cat(fine_z, dim=2)

    def _route(self, hv, page_z, fine_z):
        """Anchor routing (tao_stream.py:310-357); hv [1,1,H,P,D]."""
        b, length, heads, _, d = hv.shape
        completed, pending = len(self.pages), len(self.pending)
        coarse, _, count = routed_counts(completed, pending, self.GROUP)
        pages, ids = [], []
        chosen = None
        if coarse:
            mass = hv[..., :completed, :].sum(-1)
            chosen = topk_oldest(mass, coarse).sort(-1).values
            seg = torch.arange(self.GROUP)
            pages.append(chosen.unsqueeze(-1).expand(b, length, heads, coarse, self.GROUP)
                         .reshape(b, length, heads, coarse * self.GROUP))
            ids.append((chosen.unsqueeze(-1) * self.GROUP + seg)
                       .reshape(b, length, heads, coarse * self.GROUP))
        if pending:
            pid = torch.arange(pending).view(1, 1, 1, pending).expand(b, length, heads, pending)
            pages.append(torch.full_like(pid, completed))
            ids.append(completed * self.GROUP + pid)
        pages = torch.cat(pages, -1)
        ids = torch.cat(ids, -1)
        zc = fine_z[:, None].expand(-1, length, -1, -1, -1).gather(3, ids[..., None].expand(-1, -1, -1, -1, d))
        pzc = page_z[:, None].expand(-1, length, -1, -1, -1).gather(3, pages[..., None].expand(-1, -1, -1, -1, d))
        weight = (zc - pzc).exp().to(hv.dtype)
        channel = hv.gather(3, pages[..., None].expand(-1, -1, -1, -1, d))
        mass = (channel * weight).to(hv.dtype).sum(-1)
        selected = topk_oldest(mass, count)
        selected_id = ids.gather(-1, selected)
        self.route_ids = (chosen if coarse else pages[..., :0], selected_id)

    def _read_segment(self, raw_q, refresh):
        dtype = raw_q.dtype
        feature = self.fine_writer in FEATURE_WRITERS
        h = F.softmax(raw_q.float() if feature else raw_q, dim=-1).to(dtype)
        page_z, fine_z = self._page_tables(dtype)
        page_weight = F.softmax(page_z, dim=2).to(dtype)
        hv = (h.unsqueeze(3) * page_weight[:, None]).to(dtype)
        if self.pages and not self.coarse_index_only:
            self.coarse_parts.append(coarse_read(h, page_z[:, :, :len(self.pages)],
                                                 torch.stack(self.page_c, dim=2)))
        if refresh:
            self._route(hv[:, :1], page_z, fine_z)
        ids = self.route_ids[1].expand(-1, raw_q.shape[1], -1, -1)
        if feature:  # tao_stream.py:362-367
            d = raw_q.shape[-1]
            sel_z = fine_z[:, None].expand(-1, raw_q.shape[1], -1, -1, -1).gather(
                3, ids[..., None].expand(-1, -1, -1, -1, d))
            return feature_read(h, sel_z, ids, self.fine_c)
        return fine_read(hv, page_z, fine_z, ids, self.fine_c, self.GROUP)[-1]

    def read(self, raw_q, position):
        """_read_progressive (tao_stream.py:196-227); returns (fine, fine_on); the
        coarse read of the same segments is left in ``last_coarse`` (None when no
        page is complete or the pages are index-only)."""
        self.coarse_parts = []
        self.last_coarse = None
        if not self.pages and not self.pending:
            return torch.zeros_like(raw_q), False
        first_fine = self.serve_limit
        first_turn = first_fine + self.STAGGER * self.layer_index
        out = []
        offset = 0
        while offset < raw_q.shape[1]:
            absolute = position + offset
            refresh = (absolute == first_fine or
                       (absolute >= first_turn and (absolute - first_turn) % self.PERIOD == 0))
            nxt = (first_turn if absolute < first_turn else
                   first_turn + self.PERIOD * ((absolute - first_turn) // self.PERIOD + 1))
            count = min(raw_q.shape[1] - offset, nxt - absolute)
            out.append(self._read_segment(raw_q[:, offset:offset + count], refresh))
            if refresh:
                self.route_refreshes += 1
            offset += count
        if self.coarse_parts:
            self.last_coarse = torch.cat(self.coarse_parts, dim=1)
        return torch.cat(out, dim=1), True

    def seal(self, raw_k, v):
        """LayerState.seal/append_fine (tao_stream.py:435-512), index-only pages."""
        z, c = seal_block(raw_k, v)
        if self.fine_writer == "structured_gram_association":
            # tao_stream.py:58-61 and 463-472: z = bf16(log feature mass), C from the
            # structured inverse; square mass, cross and mass accumulate without reset
            square, cross, mass = structured_statistics(raw_k, v)
            c = structured_matrix(square, cross, mass, self.FINE)
            z = mass.log().to(raw_k.dtype)
            self.pending_mass = mass if self.pending_mass is None else self.pending_mass + mass
            self.pending_square_mass = (square if self.pending_square_mass is None
                                        else self.pending_square_mass + square)
            self.pending_cross = cross if self.pending_cross is None else self.pending_cross + cross
        elif self.fine_writer == "feature_mass_association":
            # tao_stream.py:62-65 and 463-500: z = bf16(log feature mass), C from the
            # unchecked regularised solve; mass and statistics accumulate without reset
            gram, cross, mass = association_statistics(raw_k, v, with_mass=True)
            c = association_matrix(gram, cross, unchecked=True)
            z = mass.log().to(raw_k.dtype)
            self.pending_mass = mass if self.pending_mass is None else self.pending_mass + mass
            self.pending_gram = gram if self.pending_gram is None else self.pending_gram + gram
            self.pending_cross = cross if self.pending_cross is None else self.pending_cross + cross
        elif self.fine_writer == "regularized_association":
            # tao_stream.py:72-74 and 463-475: same z, C from the regularised solve;
            # with index-only pages the statistics keep accumulating (never reset)
            gram, cross = association_statistics(raw_k, v)
            c = association_matrix(gram, cross)
            self.pending_gram = gram if self.pending_gram is None else self.pending_gram + gram
            self.pending_cross = cross if self.pending_cross is None else self.pending_cross + cross
        self.state_version += 1
        c = c.unsqueeze(2)
        self.fine_c = c if self.fine_c is None else torch.cat((self.fine_c, c), dim=2)
        self.pending.append(z)
        if len(self.pending) == self.GROUP:
            zs = torch.stack(self.pending, dim=2)
            pz = (self.pending_mass.log().to(zs.dtype) if self.fine_writer in FEATURE_WRITERS
                  else torch.logsumexp(zs, dim=2).to(zs.dtype))
            if not self.coarse_index_only:
                if self.fine_writer != "softmax":
                    raise NotImplementedError("coarse value pages are restated for the softmax writer")
                self.page_c.append(page_matrix(zs, pz, self.fine_c[:, :, -self.GROUP:]))
            self.pages.append((pz, zs))
            self.pending = []

    # -- one chunk (StreamCache.process, tao_stream.py:919-979) ----------
    def process(self, raw_q, raw_k, q, k, v):
        if self.local is None:
            ak, av, ar = k, v, raw_k
        else:
            ak = torch.cat((self.local[0], k), 1)
            av = torch.cat((self.local[1], v), 1)
            ar = torch.cat((self.local[2], raw_k), 1)
        if ak.shape[1] > self.serve_limit:
            raise ValueError("chunk crosses a fine seal boundary")
        local = local_attention(q, ak, av)
        fine, fine_on = self.read(raw_q, self.position)
        coarse = self.last_coarse
        if ak.shape[1] == self.serve_limit:
            self.fine_seal_events += 1
            self.seal(ar[:, :self.FINE], av[:, :self.FINE])
            self.local = (ak[:, -self.KEEP:].clone(), av[:, -self.KEEP:].clone(),
                          ar[:, -self.KEEP:].clone())
        else:
            self.local = (ak, av, ar)
        return local, fine, fine_on, coarse

    def step(self, q, k, v, raw_q, raw_k, fa, fb, alpha):
        """tao_attention_prefill (operator.py:70-127): chunked at seal boundaries."""
        outs = []
        start = 0
        while start < q.shape[1]:
            width = self.next_chunk(q.shape[1] - start)
            sl = slice(start, start + width)
            local, fine, fine_on, coarse = self.process(raw_q[:, sl], raw_k[:, sl], q[:, sl], k[:, sl], v[:, sl])
            outs.append(fuse_inference(raw_q[:, sl], local, fine, fa, fb, alpha, fine_on,
                                       coarse, coarse is not None))
            self.position += width
            start += width
        return torch.cat(outs, dim=1)

    # -- snapshot in the reference's dictionary format -------------------
    def export(self):
        """StreamCache.export keys (tao_stream.py:853-877)."""
        clone = lambda t: t.detach().clone()
        return {
            "layer_index": self.layer_index,
            "position": self.position,
            "local": None if self.local is None else tuple(map(clone, self.local)),
            "packed_fine_c": None if self.fine_c is None else clone(self.fine_c),
            "pages": [(clone(pz), clone(self.page_c[i]) if self.page_c else None, clone(fz))
                      for i, (pz, fz) in enumerate(self.pages)],
            "pending_z": [clone(z) for z in self.pending],
            "pending_gram": None if self.pending_gram is None else clone(self.pending_gram),
            "pending_cross": None if self.pending_cross is None else clone(self.pending_cross),
            "pending_mass": None if self.pending_mass is None else clone(self.pending_mass),
            "pending_square_mass": None if self.pending_square_mass is None else clone(self.pending_square_mass),
            "route_ids": None if self.route_ids is None else tuple(map(clone, self.route_ids)),
            "state_version": self.state_version,
            "route_refreshes": self.route_refreshes,
            "fine_seal_events": self.fine_seal_events,
        }

    @classmethod
    def from_export(cls, saved):
        config = saved.get("config", {})
        st = cls(saved["layer_index"], config.get("fine_writer", "softmax"), config.get("coarse_index_only", True))
        st.position = saved["position"]
        cpu = lambda t: t.detach().to("cpu").clone()
        st.local = None if saved["local"] is None else tuple(map(cpu, saved["local"]))
        st.fine_c = None if saved["packed_fine_c"] is None else cpu(saved["packed_fine_c"])
        st.pages = [(cpu(pz), cpu(fz)) for pz, _, fz in saved["pages"]]
        st.page_c = [] if st.coarse_index_only else [cpu(pc) for _, pc, _ in saved["pages"]]
        st.pending = [cpu(z) for z in saved["pending_z"]]
        st.pending_gram = None if saved.get("pending_gram") is None else cpu(saved["pending_gram"])
        st.pending_cross = None if saved.get("pending_cross") is None else cpu(saved["pending_cross"])
        st.pending_mass = None if saved.get("pending_mass") is None else cpu(saved["pending_mass"])
        st.pending_square_mass = (None if saved.get("pending_square_mass") is None
                                  else cpu(saved["pending_square_mass"]))
        st.route_ids = None if saved["route_ids"] is None else tuple(map(cpu, saved["route_ids"]))
        st.state_version = saved["state_version"]
        st.route_refreshes = saved.get("route_refreshes", 0)
        st.fine_seal_events = saved.get("fine_seal_events", 0)
        return st


# --------------------------------------------------------------------------
# Training read (tao_stream.py:530-787) and tao_attention (operator.py:21-54)
# --------------------------------------------------------------------------

class _SelectedRead(torch.autograd.Function):
    """selected_read.py:156-187 restated: forward N/D and the reference adjoints
    with their bf16 rounding points (dA, dhv in slot order, dw, per-tile dC)."""

    @staticmethod
    def forward(ctx, hv, w, ids, pages, fine_c):
        # hv [B,Q,H,P,D]; w [B,H,S,D]; ids/pages [B,Q,H,M]; fine_c [B,H,S,D,D]
        b, q, h, m = ids.shape
        d = hv.shape[-1]
        hvs = hv.gather(3, pages[..., None].expand(b, q, h, m, d)).float()
        ws = w[:, None].expand(b, q, h, -1, d).gather(3, ids[..., None].expand(b, q, h, m, d)).float()
        a = _r(hvs * ws)
        bi = torch.arange(b)[:, None, None, None]
        hi = torch.arange(h)[None, None, :, None]
        csel = fine_c[bi, hi, ids].float()
        num = torch.einsum("bqhmd,bqhmde->bqhe", a, csel).to(hv.dtype)
        den = _r(a.sum(-1)).sum(-1, keepdim=True).to(hv.dtype)
        ctx.save_for_backward(hv, w, ids, pages, fine_c)
        return num, den

    @staticmethod
    def backward(ctx, gn, gd):
        hv, w, ids, pages, fine_c = ctx.saved_tensors
        b, q, h, m = ids.shape
        d = hv.shape[-1]
        p = hv.shape[3]
        bi = torch.arange(b)[:, None, None, None]
        hi = torch.arange(h)[None, None, :, None]
        csel = fine_c[bi, hi, ids].float()                       # b,q,h,m,d,e
        gnf = gn.float()
        # dA = bf16(bf16(g . C^T) + gd)  (selected_read.py:55-77)
        nda = _r(torch.einsum("bqhe,bqhmde->bqhmd", gnf, csel))
        da = _r(nda + gd.float()[..., None])                      # [b,q,h,m,d] (gd [b,q,h,1])
        ws = w[:, None].expand(b, q, h, -1, d).gather(3, ids[..., None].expand(b, q, h, m, d)).float()
        hvs = hv.gather(3, pages[..., None].expand(b, q, h, m, d)).float()
        # dhv: per page, bf16 accumulation in slot order (selected_read.py:80-97)
        dhv = torch.zeros(b, q, h, p, d)
        prod = _r(da * ws)
        for slot in range(m):
            onehot = F.one_hot(pages[..., slot], p).bool()        # b,q,h,p
            dhv = torch.where(onehot[..., None], _r(dhv + prod[..., slot, None, :]), dhv)
        # dw: fp32 sum of bf16(dA*hv) over selected pairs (selected_read.py:100-122)
        prod_w = _r(da * hvs)
        dw = torch.zeros(b, h, w.shape[2], d)
        dw.index_put_((bi.expand(b, q, h, m), hi.expand(b, q, h, m), ids), prod_w, accumulate=True)
        # dC: per fine, bf16(sum over this example's pairs of a^T g) (selected_read.py:125-153)
        a = _r(hvs * ws)
        outer = torch.einsum("bqhmd,bqhe->bqhmde", a, gnf)
        dc = torch.zeros(b, h, fine_c.shape[2], d, d)
        dc.index_put_((bi.expand(b, q, h, m), hi.expand(b, q, h, m), ids), outer, accumulate=True)
        dc = _r(dc)
        return dhv.to(hv.dtype), dw.to(w.dtype), None, None, dc.to(fine_c.dtype)


def _local_training(q, k, v, fine=256, keep=512):
    """_local_training_corrected_4k (tao_stream.py:760-787)."""
    b, total, heads, d = q.shape
    if total < 3 * fine or total % fine:
        parts = []
        for start in range(0, total, fine):
            end = min(total, start + fine)
            old = max(0, start - keep)
            parts.append(local_attention(q[:, start:end], k[:, old:end], v[:, old:end]))
        return torch.cat(parts, dim=1)
    first = local_attention(q[:, :256], k[:, :256], v[:, :256])
    second = local_attention(q[:, 256:512], k[:, :512], v[:, :512])
    n = total // 256 - 2
    query = q[:, 512:].reshape(b * n, 256, heads, d)
    keys = k.unfold(1, 768, 256).permute(0, 1, 4, 2, 3).reshape(b * n, 768, heads, d)
    values = v.unfold(1, 768, 256).permute(0, 1, 4, 2, 3).reshape(b * n, 768, heads, d)
    later = local_attention(query, keys, values)
    return torch.cat((first, second, later.reshape(b, total - 512, heads, d)), dim=1)


def _tile_read(query, page_z, fine_z, fine_c, completed, pending, group=8, page_c=None, feature=False):
    """_read_training_group for one 256-query tile (tao_stream.py:596-665);
    with ``page_c`` (the completed pages' matrices) also the coarse read
    (tao_stream.py:611-617); with ``feature`` (the feature-read writers) h is the
    fp32 softmax rounded once and the read is the feature-mass read of the selected
    fines, no denominator (tao_stream.py:600-601, 658-661).  Returns (fine, selected
    ids, coarse or None)."""
    b, length, heads, d = query.shape
    dt = query.dtype
    h = F.softmax(query.float() if feature else query, dim=-1).to(dt)
    coarse_out = None
    if page_c is not None and completed:
        coarse_out = coarse_read(h, page_z[:, :, :completed], page_c[:, :, :completed])
    page_weight = F.softmax(page_z, dim=2).to(dt)
    hv = (h.unsqueeze(3) * page_weight[:, None]).to(dt)
    coarse, _, count = routed_counts(completed, pending, group)
    visible = completed * group + pending
    with torch.no_grad():
        cand_pages, cand_ids = [], []
        if coarse:
            mass = hv[..., :completed, :].sum(-1)
            chosen = topk_oldest(mass, coarse).sort(-1).values
            seg = torch.arange(group)
            cand_pages.append(chosen.unsqueeze(-1).expand(b, length, heads, coarse, group)
                              .reshape(b, length, heads, coarse * group))
            cand_ids.append((chosen.unsqueeze(-1) * group + seg).reshape(b, length, heads, coarse * group))
        if pending:
            pid = torch.arange(pending).view(1, 1, 1, pending).expand(b, length, heads, pending)
            cand_pages.append(torch.full_like(pid, completed))
            cand_ids.append(completed * group + pid)
        cand_pages = torch.cat(cand_pages, -1)
        cand_ids = torch.cat(cand_ids, -1)
    fine_page = torch.arange(fine_z.shape[2]) // group
    seg_w = (fine_z - page_z.index_select(2, fine_page)).exp().to(dt)
    with torch.no_grad():
        hvd, wd = hv.detach(), seg_w.detach()
        u = cand_ids.shape[-1]
        ch = (hvd.gather(3, cand_pages[..., None].expand(b, length, heads, u, d)).float()
              * wd[:, None].expand(b, length, heads, -1, d).gather(3, cand_ids[..., None].expand(b, length, heads, u, d)).float()).to(BF16)
        scores = ch.sum(-1).masked_fill(cand_ids >= visible, -torch.inf)
        sel = topk_oldest(scores, count)
        sel_id = cand_ids.gather(-1, sel)
        sel_page = cand_pages.gather(-1, sel)
    if feature:   # the selected z by expand + gather, as the reference (its adjoint sums in fp32)
        sel_z = fine_z[:, None].expand(-1, length, -1, -1, -1).gather(3, sel_id.unsqueeze(-1).expand(-1, -1, -1, -1, d))
        return feature_read(h, sel_z, sel_id, fine_c), sel_id, coarse_out
    num, den = _SelectedRead.apply(hv, seg_w, sel_id, sel_page, fine_c)
    return (num / den).to(dt), sel_id, coarse_out


def training_page_matrices(fine_z, fine_c, group=8):
    """Coarse page matrices of every completed page in training
    (_training_metadata with n == group, tao_stream.py:552-573): the page's
    log-partition, then the page matrix as in streaming."""
    b, heads, s, d = fine_z.shape
    full = s // group
    if not full:
        return None
    zc = fine_z[:, :, :full * group].reshape(b, heads, full, group, d)
    pz = torch.logsumexp(zc, dim=3).to(fine_z.dtype)
    cc = fine_c[:, :, :full * group].reshape(b, heads, full, group, d, d)
    weight = (zc - pz.unsqueeze(3)).exp().to(fine_z.dtype)
    with torch.autocast(device_type="cpu", enabled=False):
        return torch.einsum("bhpsd,bhpsde->bhpde", weight, cc).to(fine_z.dtype)


def training_read(raw_q, raw_k, v, q, k, fine=256, group=8, keep_ids=False, writer="softmax",
                  coarse_index_only=True):
    """read_training (tao_stream.py:668-757) with route_interval=1; returns
    (local, fine, [selected ids per tile]); with coarse_index_only=False also the
    coarse value read as a fourth element (zeros before the first complete page)."""
    local = _local_training(q, k, v)
    b, total, heads, d = q.shape
    if total <= keep_plus(fine):
        if not coarse_index_only:
            return local, torch.zeros_like(local), [], torch.zeros_like(local)
        return local, torch.zeros_like(local), []
    feature = writer in FEATURE_WRITERS
    if feature:
        fine_z, fine_c, fine_mass = seal_all_feature(raw_k, v, writer, fine)
    else:
        fine_z, fine_c = seal_all(raw_k, v, fine, writer)
    if not coarse_index_only and writer != "softmax":
        raise NotImplementedError("coarse value pages are restated for the softmax writer")
    page_c = None if coarse_index_only else training_page_matrices(fine_z, fine_c, group)
    fine_parts, ids, coarse_parts = [], [], []
    for tile, query in enumerate(raw_q.split(fine, dim=1)):
        visible = max(0, tile - 2)
        if not visible:
            fine_parts.append(torch.zeros_like(query))
            coarse_parts.append(torch.zeros_like(query))
            continue
        completed, pending = divmod(visible, group)
        pz = []
        if feature:   # page z = bf16(log of the page's fp32 mass summed in fine order)
            if completed:
                mc = fine_mass[:, :, :completed * group].reshape(b, heads, completed, group, d)
                pz.append(chronological_sum(mc, 3).log().to(fine_z.dtype))
            if pending:
                mp = fine_mass[:, :, completed * group:visible].reshape(b, heads, 1, pending, d)
                pz.append(chronological_sum(mp, 3).log().to(fine_z.dtype))
        else:
            if completed:
                zc = fine_z[:, :, :completed * group].reshape(b, heads, completed, group, d)
                pz.append(torch.logsumexp(zc, dim=3).to(fine_z.dtype))
            if pending:
                zp = fine_z[:, :, completed * group:visible].reshape(b, heads, 1, pending, d)
                pz.append(torch.logsumexp(zp, dim=3).to(fine_z.dtype))
        page_z = torch.cat(pz, dim=2)
        out, sel, coarse = _tile_read(query, page_z, fine_z[:, :, :visible], fine_c[:, :, :visible],
                                      completed, pending, group, page_c, feature=feature)
        fine_parts.append(out)
        coarse_parts.append(torch.zeros_like(query) if coarse is None else coarse)
        if keep_ids:
            ids.append(sel)
    if not coarse_index_only:
        return local, torch.cat(fine_parts, dim=1), ids, torch.cat(coarse_parts, dim=1)
    return local, torch.cat(fine_parts, dim=1), ids


def training_routes(raw_q, raw_k, v, fine=256, group=8):
    """The routing decisions of read_training (tao_stream.py:596-665) for every
    256-query tile, with the scores behind them, so a test can tell a real routing
    difference from a near-tie: per tile a dict with ``sel`` [B,L,H,M] (selected
    fine ids in rank order, as ``_tile_read``), ``page_mass`` [B,L,H,completed]
    (bf16 sum_d hv of each completed page), ``chosen`` [B,L,H,K] (pages kept) and
    ``fine_score`` [B,L,H,visible] (bf16 sum_d bf16(hv[page] * w) of every visible
    fine, candidate or not: the score it would have as a candidate)."""
    b, total, heads, d = raw_q.shape
    if total <= keep_plus(fine):
        return []
    fine_z, _ = seal_all(raw_k, v, fine)
    dt = raw_q.dtype
    tiles = []
    for tile, query in enumerate(raw_q.split(fine, dim=1)):
        visible = max(0, tile - 2)
        if not visible:
            continue
        completed, pending = divmod(visible, group)
        pz = []
        if completed:
            zc = fine_z[:, :, :completed * group].reshape(b, heads, completed, group, d)
            pz.append(torch.logsumexp(zc, dim=3).to(dt))
        if pending:
            zp = fine_z[:, :, completed * group:visible].reshape(b, heads, 1, pending, d)
            pz.append(torch.logsumexp(zp, dim=3).to(dt))
        page_z = torch.cat(pz, dim=2)
        length = query.shape[1]
        h = F.softmax(query, dim=-1).to(dt)
        hv = (h.unsqueeze(3) * F.softmax(page_z, dim=2).to(dt)[:, None]).to(dt)
        coarse, _, count = routed_counts(completed, pending, group)
        fz = fine_z[:, :, :visible]
        fine_page = torch.arange(visible) // group
        w = (fz - page_z.index_select(2, fine_page)).exp().to(dt)            # [B,H,V,D]
        hv_f = hv.index_select(3, fine_page)                                   # [B,L,H,V,D]
        score = (hv_f.float() * w[:, None].float()).to(BF16).sum(-1)           # [B,L,H,V]
        info = dict(tile=tile, coarse=coarse, count=count, completed=completed, pending=pending,
                    fine_score=score.float())
        ids = []
        if coarse:
            mass = hv[..., :completed, :].sum(-1)
            chosen = topk_oldest(mass, coarse).sort(-1).values
            info["page_mass"] = mass.float()
            info["chosen"] = chosen
            ids.append((chosen.unsqueeze(-1) * group + torch.arange(group)).reshape(b, length, heads, -1))
        if pending:
            ids.append((completed * group + torch.arange(pending)).view(1, 1, 1, pending).expand(b, length, heads,
                                                                                                 pending))
        cand = torch.cat(ids, -1)
        cand_score = score.gather(-1, cand)
        info["sel"] = cand.gather(-1, topk_oldest(cand_score, count))
        tiles.append(info)
    return tiles


def keep_plus(fine):
    return 512 + fine


def fuse_training(local, raw_q, fine, fine_present, fa, fb, alpha, coarse=None, coarse_present=None):
    """operator._fuse_training (operator.py:21-39); the coarse term is absent with
    index-only pages (coarse=None)."""
    dtype = raw_q.dtype
    score = (fa.to(dtype) * raw_q.unsqueeze(-1)).to(dtype)
    score = (score + fb.to(dtype)).to(dtype)
    if coarse_present is None:
        coarse_present = torch.zeros_like(fine_present)
    count = fine_present.to(torch.int32) + coarse_present.to(torch.int32)
    local_bias = count.clamp_min(1).to(dtype).log().to(dtype)
    score = torch.stack(((score[..., 0] + local_bias).to(dtype), score[..., 1], score[..., 2]), -1)
    score = torch.stack((score[..., 0], score[..., 1].masked_fill(~coarse_present, -torch.inf),
                         score[..., 2].masked_fill(~fine_present, -torch.inf)), -1)
    rho = F.softmax(score, dim=-1).to(dtype)
    gain = torch.full((), 2 * alpha, dtype=dtype)
    if coarse is None:
        coarse = torch.zeros_like(local)
    lt = (rho[..., 0] * (2 * local).to(dtype)).to(dtype)
    ct = (rho[..., 1] * (gain * coarse).to(dtype)).to(dtype)
    ft = (rho[..., 2] * (gain * fine).to(dtype)).to(dtype)
    fused = ((lt + ct).to(dtype) + ft).to(dtype)
    return torch.where(coarse_present | fine_present, fused, local)


def tao_attention(q, k, v, raw_q, raw_k, fa, fb, alpha, writer="softmax", coarse_index_only=True):
    """operator.tao_attention (operator.py:42-54).  ``alpha`` may be a float or a
    per-head sequence (heads are independent, so per-head alpha equals one
    reference call per head slice).  coarse_index_only=False adds the coarse value
    read, present from position 512 + 8 * 256 on (config.first_coarse)."""
    coarse = coarse_present = None
    if coarse_index_only:
        local, fine, _ = training_read(raw_q, raw_k, v, q, k, writer=writer)
    else:
        local, fine, _, coarse = training_read(raw_q, raw_k, v, q, k, writer=writer, coarse_index_only=False)
    positions = torch.arange(q.shape[1])[None, :, None, None]
    present = positions >= 768
    if not coarse_index_only:
        coarse_present = positions >= 512 + 8 * 256
    if isinstance(alpha, (int, float)):
        return fuse_training(local, raw_q, fine, present, fa, fb, alpha, coarse, coarse_present)
    outs = [fuse_training(local[:, :, i:i + 1], raw_q[:, :, i:i + 1], fine[:, :, i:i + 1],
                          present, fa[i:i + 1], fb[i:i + 1], float(alpha[i]),
                          None if coarse is None else coarse[:, :, i:i + 1], coarse_present)
            for i in range(q.shape[2])]
    return torch.cat(outs, dim=2)
