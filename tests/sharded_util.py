"""Test helpers for the row-sharded pair stack.

``OraclePhases`` is a CPU stand-in for ``fireprot_b200.sharded.CudaPhases``:
the same phase methods with the oracle's float64 math on plain layouts, so
the orchestration (shard plan, collective sequence, transposes, ragged and
empty ranks) runs on gloo ranks without a GPU. ``ThreadComm`` emulates a
process group of ``world`` threads in one process (tensor copies between the
threads at each collective), which lets one GPU run several ranks' phase
kernels; no kernel ever waits on another.
"""
import math
import threading

import torch

from oracle import pairformer_oracle as O


def _ln(x, w, b):
    return O.layer_norm(x, w.to(x.dtype), b.to(x.dtype))


def _d(t):
    return None if t is None else t.detach().to("cpu", torch.float64)


class OraclePhases:
    def __init__(self):
        self.calls = []

    def check(self):
        pass

    # TriMul: a/b planes are [plane_rows][cols][128] float64
    def trimul_proj(self, z_loc, mask, shard, outgoing, w):
        self.calls.append("trimul_proj")
        n, rows, r0 = shard.n, shard.rows, shard.r0
        if not outgoing and rows == 0:
            return None, None, 0
        zl = _d(z_loc[:rows])
        zn = _ln(zl, _d(w["ln_in_w"]), _d(w["ln_in_b"]))
        a = torch.sigmoid(zn @ _d(w["w_a_g"]).T) * (zn @ _d(w["w_a_p"]).T)
        b = torch.sigmoid(zn @ _d(w["w_b_g"]).T) * (zn @ _d(w["w_b_p"]).T)
        if mask is not None:
            m = _d(mask)[r0:r0 + rows, :, None]
            a, b = a * m, b * m
        if outgoing:
            pa = torch.zeros(shard.chunk, n, 128, dtype=torch.float64)
            pb = torch.zeros(shard.chunk, n, 128, dtype=torch.float64)
            pa[:rows], pb[:rows] = a, b
            return [pa], [pb], None
        return [a.transpose(0, 1).contiguous()], [b.transpose(0, 1).contiguous()], None

    def new_x(self, rows, shard, device):
        return torch.zeros(rows, shard.n, 128, dtype=torch.float64)

    def trimul_contract_out(self, a, b_full, shard, ld):
        self.calls.append("trimul_contract_out")
        x = self.new_x(shard.chunk, shard, None)
        bf = b_full[0].reshape(shard.world * shard.chunk, shard.n, 128)[:shard.n]
        x[:shard.rows] = torch.einsum("ikc,jkc->ijc", a[0][:shard.rows], bf)
        return x

    def trimul_contract_in(self, a, b, shard, ld, device):
        self.calls.append("trimul_contract_in")
        x = self.new_x(shard.world * shard.chunk, shard, device)
        if shard.rows:
            x[:shard.n] = torch.einsum("ikc,jkc->ijc", a[0], b[0])
        return x

    def trimul_finish(self, z_loc, shard, x_loc, w, add):
        self.calls.append("trimul_finish")
        rows = shard.rows
        if rows == 0:
            return
        zl = _d(z_loc[:rows])
        zn = _ln(zl, _d(w["ln_in_w"]), _d(w["ln_in_b"]))
        x = _ln(x_loc[:rows], _d(w["ln_out_w"]), _d(w["ln_out_b"])) @ _d(w["w_z"]).T
        delta = torch.sigmoid(zn @ _d(w["w_g"]).T) * x
        z_loc[:rows] = (zl + delta if add else delta).to(z_loc.dtype)

    # TriMul, channel groups: planes [128][rows_p][cols] float64
    def trimul_proj_groups(self, z_loc, mask, shard, outgoing, w):
        self.calls.append("trimul_proj_groups")
        n, rows, chunk = shard.n, shard.rows, shard.chunk
        pa = torch.zeros(128, chunk, n, dtype=torch.float64) if outgoing else \
            torch.zeros(128, n, chunk, dtype=torch.float64)
        pb = torch.zeros_like(pa)
        if rows:
            a, b, _ = self.trimul_proj(z_loc, mask, shard, True, w)
            self.calls.pop()
            a, b = a[0][:rows].permute(2, 0, 1), b[0][:rows].permute(2, 0, 1)  # [c][i][k]
            if outgoing:
                pa[:, :rows], pb[:, :rows] = a, b
            else:
                pa[:, :, :rows], pb[:, :, :rows] = a.transpose(1, 2), b.transpose(1, 2)
        return pa, pb, (n if outgoing else chunk)

    def trimul_contract_groups(self, ra, rb, shard, outgoing, ld):
        self.calls.append("trimul_contract_groups")
        W, n, chunk = shard.world, shard.n, shard.chunk
        G = 128 // W
        if outgoing:
            def op(r):
                return r.view(W, G, chunk, n).transpose(0, 1).reshape(G, W * chunk, n)[:, :n]
        else:
            def op(r):
                return r.view(W, G, n, chunk).permute(1, 2, 0, 3).reshape(G, n, W * chunk)
        xg = torch.zeros(W * chunk, n, G, dtype=torch.float64)
        xg[:n] = torch.einsum("cik,cjk->ijc", op(ra), op(rb))
        return xg

    def trimul_ungroup_x(self, rx, shard):
        W, chunk, n = shard.world, shard.chunk, shard.n
        return rx.view(W, chunk, n, 128 // W).permute(1, 2, 0, 3).reshape(chunk, n, 128)

    # TriAttn: bias buffer [world*chunk][4][n] (j-major), state = mask rows
    def triattn_bias_buffer(self, shard, device):
        return torch.zeros(shard.world * shard.chunk, 4, shard.n, dtype=torch.float64)

    def triattn_proj(self, z_loc, mask, shard, w, bias_full):
        self.calls.append("triattn_proj")
        rows, r0 = shard.rows, shard.r0
        if rows == 0:
            return None
        zn = _ln(_d(z_loc[:rows]), _d(w["ln_w"]), _d(w["ln_b"]))
        bias_full[r0:r0 + rows] = (zn @ _d(w["w_bias"]).T).permute(0, 2, 1)
        return None if mask is None else _d(mask)[r0:r0 + rows]

    def triattn_finish(self, z_loc, shard, with_mask, bias_full, w, state):
        self.calls.append("triattn_finish")
        rows, n = shard.rows, shard.n
        if rows == 0:
            return
        zl = _d(z_loc[:rows])
        zn = _ln(zl, _d(w["ln_w"]), _d(w["ln_b"]))
        H, dh = 4, 32
        q = (zn @ _d(w["w_q"]).T).reshape(rows, n, H, dh).permute(0, 2, 1, 3) / math.sqrt(dh)
        k = (zn @ _d(w["w_k"]).T).reshape(rows, n, H, dh).permute(0, 2, 1, 3)
        v = (zn @ _d(w["w_v"]).T).reshape(rows, n, H, dh).permute(0, 2, 1, 3)
        tri = bias_full[:n].permute(1, 0, 2).unsqueeze(0)  # [1, h, j, k]
        biases = []
        if with_mask:
            biases.append((O.MASK_INF * (state - 1.0))[:, None, None, :])
        biases.append(tri)
        o = O.attention_core(q, k, v, biases).permute(0, 2, 1, 3).reshape(rows, n, H * dh)
        g = zn @ _d(w["w_g"]).T
        if w.get("b_g") is not None:
            g = g + _d(w["b_g"])
        out = (torch.sigmoid(g) * o) @ _d(w["w_o"]).T
        if w.get("b_o") is not None:
            out = out + _d(w["b_o"])
        z_loc[:rows] = (zl + out).to(z_loc.dtype)

    def transition(self, z_loc, shard, w):
        self.calls.append("transition")
        rows = shard.rows
        if rows == 0:
            return
        zl = _d(z_loc[:rows])
        p = O.TransitionParams(**{k: _d(w[k]) for k in ("ln_w", "ln_b", "w_a", "w_b", "w_out")})
        z_loc[:rows] = (zl + O.pair_transition(zl, p)).to(z_loc.dtype)

    def single_block(self, s, z_loc, mask, shard, w):
        """Query rows of the rank: the full oracle on a pair tensor holding
        only the rank's rows (query i reads pair row i alone)."""
        self.calls.append("single_block")
        n, rows, r0 = shard.n, shard.rows, shard.r0
        if rows == 0:
            return
        z = torch.zeros(n, n, 128, dtype=torch.float64)
        z[r0:r0 + rows] = _d(z_loc[:rows])
        out = O.single_block(_d(s), z, _d(mask), oracle_single_params(w))
        s[r0:r0 + rows] = out[r0:r0 + rows].to(s.dtype)


def single_weight_dict(p: "O.SingleBlockParams") -> dict:
    """``PairformerSingleBlock.weight_dict()`` keys from oracle parameters."""
    d = {k: getattr(p, k) for k in ("ln_a_w", "ln_a_b", "w_q", "b_q", "w_k", "w_v", "w_g",
                                    "w_o", "ln_z_w", "ln_z_b", "w_z")}
    t = p.transition
    d.update(tr_ln_w=t.ln_w, tr_ln_b=t.ln_b, tr_w_a=t.w_a, tr_w_b=t.w_b, tr_w_out=t.w_out)
    return d


def oracle_single_params(w: dict, heads: int = 16, head_dim: int = 24,
                         dtype=torch.float64) -> "O.SingleBlockParams":
    """Inverse of ``single_weight_dict`` (CPU copies in ``dtype``)."""
    def c(t):
        return t.detach().to("cpu", dtype)
    tr = O.TransitionParams(ln_w=c(w["tr_ln_w"]), ln_b=c(w["tr_ln_b"]), w_a=c(w["tr_w_a"]),
                            w_b=c(w["tr_w_b"]), w_out=c(w["tr_w_out"]))
    return O.SingleBlockParams(heads=heads, head_dim=head_dim, transition=tr, **{
        k: c(w[k]) for k in ("ln_a_w", "ln_a_b", "w_q", "b_q", "w_k", "w_v", "w_g", "w_o",
                             "ln_z_w", "ln_z_b", "w_z")})


def oracle_weight_dicts(p: "O.PairBlockParams") -> dict:
    """``sharded_pair_block`` weight dicts from oracle block parameters."""
    def tm(t):
        return {k: getattr(t, k) for k in ("ln_in_w", "ln_in_b", "w_a_p", "w_a_g", "w_b_p",
                                          "w_b_g", "w_g", "ln_out_w", "ln_out_b", "w_z")}

    def ta(t):
        return {k: getattr(t, k) for k in ("ln_w", "ln_b", "w_q", "w_k", "w_v", "w_bias", "w_g",
                                          "b_g", "w_o", "b_o")}
    tr = p.transition
    return {"tri_mul_out": tm(p.tri_mul_out), "tri_mul_in": tm(p.tri_mul_in),
            "tri_att_start": ta(p.tri_att_start), "tri_att_end": ta(p.tri_att_end),
            "pair_transition": {k: getattr(tr, k) for k in ("ln_w", "ln_b", "w_a", "w_b",
                                                            "w_out")}}


class ThreadComm:
    """One rank's view of an in-process group of ``world`` threads."""

    class Hub:
        def __init__(self, world):
            self.world = world
            self.barrier = threading.Barrier(world, timeout=120)
            self.slots = [None] * world

    def __init__(self, hub, rank):
        self.hub, self.rank, self.world = hub, rank, hub.world

    def _exchange(self, inp):
        h = self.hub
        h.slots[self.rank] = inp
        h.barrier.wait()
        got = list(h.slots)
        h.barrier.wait()
        return got

    def all_gather(self, out, inp):
        got = self._exchange(inp)
        out.view(self.world, -1).copy_(torch.stack([g.reshape(-1) for g in got]))

    def reduce_scatter(self, out, inp):
        got = self._exchange(inp)
        acc = None
        for g in got:
            part = g.view(self.world, -1)[self.rank].to(torch.float64)
            acc = part if acc is None else acc + part
        out.view(-1).copy_(acc.to(out.dtype))

    def all_to_all(self, out, inp):
        got = self._exchange(inp)
        dst = out.view(self.world, -1)
        for s, g in enumerate(got):
            dst[s].copy_(g.view(self.world, -1)[self.rank])


def run_threads(world, fn):
    """Run ``fn(rank, comm)`` on ``world`` threads; re-raise the first error."""
    hub = ThreadComm.Hub(world)
    results, errors = [None] * world, []

    def body(r):
        try:
            results[r] = fn(r, ThreadComm(hub, r))
        except BaseException as e:  # noqa: BLE001 - surfaced below
            errors.append(e)
            hub.barrier.abort()

    threads = [threading.Thread(target=body, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    if errors:
        raise errors[0]
    return results
