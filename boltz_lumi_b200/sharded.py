"""Row-sharded Pairformer block for large N (one process per GPU).

The pair tensor z [N, N, 128] (fp32) is split by rows across P ranks: rank r
holds rows I_r = [r N/P, (r + 1) N/P).  Every op then runs the same kernels as
the single-GPU path on its slab, with the exchanges the op needs:

* Triangle multiplication, channel-sharded products (P divides 128): each
  rank projects its rows into channel planes a, b ([c][row][col], rows I_r);
  one all_to_all per operand regroups them by channel, so rank r holds all
  rows of the planes of its channels C_r (128 / P of them); it computes
  O_c = a_c b_c^T (outgoing) or a_c^T b_c (incoming: the contraction runs
  over the row index, which the channel split makes local) for every pair,
  and one all_to_all of O returns the rows I_p of all channels to rank p.
  Per op a rank receives 3 (P - 1) / P^2 of a 1 GiB plane set at N = 2048
  (a, b, O), and the incoming op needs no row <-> column transpose of z.
  With P = 2 or 3 the outgoing op instead all-gathers b (less data there):
  O_c[I_r, :] = a_r b_c^T as one per-channel GEMM per source rank, and P = 3
  runs the incoming op as the outgoing form on z^T (column layout) with the
  operand halves swapped:
  z[i, j] += sum_k a[k, i] b[k, j]  ==  z'[j, i] += sum_k b'[j, k] a'[i, k],  z' = z^T.
* TriangleAttentionStartingNode (row layout): local rows; the triangle bias
  [4, N, N] (one row block per rank) is all-gathered.
* TriangleAttentionEndingNode: the starting form on z^T (column layout), as
  upstream runs it (triangle.py:131 transposes the pair axes).
* Transition: pointwise per pair row, no exchange.
* Single track: sharded by query rows.  The pair bias rows of a rank's own
  queries are local (its z rows); each rank attends with its queries over all
  tokens, applies proj_o and transition_s to its rows, and one all_gather of
  the updated s rows (N x c_s fp32) rebuilds s on every rank.

Layout changes row <-> column are one all_to_all of the slab (each rank keeps
1/P and sends (P - 1)/P of it) plus a local block transpose.  The collectives
go through a small `Comm` interface: `TorchComm` wraps torch.distributed
(NCCL over NVLink on a B200 box, gloo on CPU); `ThreadComm` emulates P ranks as
threads of one process on one GPU, which is how the decomposition is checked
against the unsharded block without several GPUs.
"""

import threading

import torch

from . import _lib, forwards, kernels
from ._lib import call, stream_of
from .forwards import _BF16, _Q_SCALE, _f32

__all__ = ["Comm", "SingleComm", "TorchComm", "ThreadComm", "rows_to_columns", "ShardedPairformer"]


# ---------------------------------------------------------------------------
# Collectives
# ---------------------------------------------------------------------------
class _Ready:
    """A collective that has already completed."""

    def __init__(self, value):
        self.value = value

    def wait(self):
        return self.value


class Comm:
    """The two collectives the sharded block needs."""

    rank = 0
    world = 1

    def all_gather(self, t):
        """[world, *t.shape]: entry p is rank p's tensor."""
        raise NotImplementedError

    def all_gather_async(self, t):
        """Start an all_gather; ``.wait()`` returns its result and orders the
        current stream after it (here: completed at once)."""
        return _Ready(self.all_gather(t))

    def all_to_all(self, t):
        """t is [world, ...] with chunk p addressed to rank p; returns [world, ...]
        with chunk p received from rank p."""
        raise NotImplementedError


class TorchComm(Comm):
    """torch.distributed collectives on an initialised process group."""

    def __init__(self, group=None):
        import torch.distributed as dist

        self.dist, self.group = dist, group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def all_gather(self, t):
        t = t.contiguous()
        flat = t.view(-1)
        out = torch.empty(self.world * flat.numel(), dtype=t.dtype, device=t.device)
        self.dist.all_gather_into_tensor(out, flat, group=self.group)
        return out.view((self.world,) + tuple(t.shape))

    def all_to_all(self, t):
        t = t.contiguous()
        out = torch.empty_like(t)
        self.dist.all_to_all_single(out, t, group=self.group)
        return out

    def all_gather_async(self, t):
        """NCCL runs the gather on its own stream; compute queued on the
        current stream before ``.wait()`` overlaps it."""
        t = t.contiguous()
        flat = t.view(-1)
        out = torch.empty(self.world * flat.numel(), dtype=t.dtype, device=t.device)
        work = self.dist.all_gather_into_tensor(out, flat, group=self.group, async_op=True)
        shape = (self.world,) + tuple(t.shape)

        class _Pending:
            def wait(self):
                work.wait()
                return out.view(shape)

        return _Pending()


class SingleComm(Comm):
    """World of one (no process group needed)."""

    def all_gather(self, t):
        return t.contiguous().unsqueeze(0)

    def all_to_all(self, t):
        return t.contiguous()


class _ThreadHub:
    def __init__(self, world):
        self.world = world
        self.slots = [None] * world
        self.barrier = threading.Barrier(world, timeout=300)  # a rank that dies breaks it instead of hanging


class ThreadComm(Comm):
    """P virtual ranks as threads of one process sharing one device.  Each
    exchange synchronises the device, so it is for checking the decomposition,
    not for speed."""

    def __init__(self, hub, rank):
        self.hub, self.rank, self.world = hub, rank, hub.world

    @staticmethod
    def group(world):
        hub = _ThreadHub(world)
        return [ThreadComm(hub, r) for r in range(world)]

    def _exchange(self, t):
        if t.is_cuda:
            torch.cuda.synchronize()
        self.hub.slots[self.rank] = t
        self.hub.barrier.wait()
        peers = list(self.hub.slots)
        return peers

    def _done(self):
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        self.hub.barrier.wait()

    def all_gather(self, t):
        peers = self._exchange(t.contiguous())
        out = torch.stack(peers)
        self._done()
        return out

    def all_to_all(self, t):
        peers = self._exchange(t.contiguous())
        out = torch.stack([peers[p][self.rank] for p in range(self.world)])
        self._done()
        return out


# ---------------------------------------------------------------------------
# Layout
# ---------------------------------------------------------------------------
def rows_to_columns(slab, comm):
    """Row slab [n_loc, N, C] of X (rows I_r) -> row slab of X^T (rows I_r of X^T,
    i.e. columns I_r of X).  Applying it twice returns the original layout."""
    n_loc, n, c = slab.shape
    world = comm.world
    send = slab.view(n_loc, world, n_loc, c).permute(1, 0, 2, 3)  # chunk p = X[I_r, I_p]
    recv = comm.all_to_all(send)  # chunk p = X[I_p, I_r]
    return recv.permute(2, 0, 1, 3).reshape(n_loc, n, c).contiguous()  # [j in I_r][i][c]


def _gather_rows(local, comm):
    """[..., n_loc, W] per rank -> [..., N, W] (row blocks concatenated in rank order)."""
    g = comm.all_gather(local)  # [P, ..., n_loc, W]
    lead = g.dim() - 3
    perm = list(range(1, 1 + lead)) + [0, lead + 1, lead + 2]
    out = g.permute(*perm)
    return out.reshape(*out.shape[:lead], out.shape[lead] * out.shape[lead + 1], out.shape[-1])


# ---------------------------------------------------------------------------
# Per-op slab forwards (the single-GPU kernels on [n_loc, N] row slabs)
# ---------------------------------------------------------------------------
def _plane_gemm(a, a_mn, b, b_mn, out, m, n, k, stream):
    """out[c][:m, :n] = bf16(A_c B_c^T) (fp32 accumulation) for every channel c of
    the strided plane views a ([cg, m, k] K-major, or [cg, k, m] with a_mn) and
    b ([cg, n, k], or [cg, k, n] with b_mn); out is [cg, m, >= n]."""
    call("bl_batched_gemm", a.data_ptr(), a_mn, a.stride(1), a.stride(0), b.data_ptr(), b_mn, b.stride(1),
         b.stride(0), out.data_ptr(), out.stride(1), out.stride(0), out.shape[0], m, n, k, None, stream)


def _channel_products(rows_op, cols_op, n, comm, incoming, stream):
    """Per-channel products of the row-sharded planes, computed channel-sharded.

    rows_op / cols_op: this rank's planes [128, n_loc, n_pad] (rows I_r).  Returns
    prod [128, n_loc, n_pad]: O_c[i in I_r, j] for every channel, with
    outgoing O_c = A_c B_c^T (planes [i][k]) and incoming O_c = A_c^T B_c (planes
    [k][i], the contraction over the sharded row index)."""
    world = comm.world
    cg, n_loc, n_pad = 128 // world, rows_op.shape[1], rows_op.shape[2]
    # Chunk p of the send buffer = channels C_p of my rows; chunk p received =
    # rank p's rows I_p of my channels C_r.
    a = comm.all_to_all(rows_op.reshape(world, cg, n_loc, n_pad))
    b = comm.all_to_all(cols_op.reshape(world, cg, n_loc, n_pad))
    b_all = b.permute(1, 0, 2, 3).reshape(cg, n, n_pad)  # [c][row in 0..N)[col]
    del b
    if incoming:
        a_all = a.permute(1, 0, 2, 3).reshape(cg, n, n_pad)  # [c][k][i]
        del a
    out = torch.empty(world, cg, n_loc, n_pad, device=rows_op.device, dtype=_BF16)
    for p in range(world):
        # out[p] = O_c[i in I_p, all j] for c in C_r: sent back to rank p.
        if incoming:  # A_c^T restricted to columns I_p (MN-major)
            _plane_gemm(a_all[:, :, p * n_loc:(p + 1) * n_loc], 1, b_all, 1, out[p], n_loc, n, n, stream)
        else:  # rank p's rows of A_c (K-major)
            _plane_gemm(a[p], 0, b_all, 0, out[p], n_loc, n, n, stream)
    del b_all
    return comm.all_to_all(out).reshape(128, n_loc, n_pad)  # chunk p = channels C_p of my rows


def _channel_split(comm):
    return comm.world > 1 and 128 % comm.world == 0


def _trimul_slab(module, x, mask_rows, comm, swap, incoming=False):
    """z_slab += triangle multiplication of `module` on the row slab x [n_loc, N, 128]
    (fp32, updated in place).  incoming=False: the outgoing form (`swap`
    exchanges the two operand halves: the incoming op on the transposed tensor);
    incoming=True: the incoming op on the row slab itself (channel-sharded
    products only)."""
    n_loc, n = x.shape[0], x.shape[1]
    n_pad = forwards._pad8(n)
    w = forwards._multiplication_weights(module)
    stream = stream_of(x)
    xn = torch.empty(n_loc * n, 128, device=x.device, dtype=_BF16)
    planes = torch.empty(256, n_loc, n_pad, device=x.device, dtype=_BF16)
    call("bl_trimul_projection", x.data_ptr(), n, n_loc, _f32(module.norm_in.weight).data_ptr(),
         _f32(module.norm_in.bias).data_ptr(), float(module.norm_in.eps), w["w_in"].data_ptr(),
         mask_rows.data_ptr(), planes.data_ptr(), n_pad, xn.data_ptr(), stream)
    rows_op, cols_op = (planes[128:], planes[:128]) if swap else (planes[:128], planes[128:])
    if incoming or (_channel_split(comm) and comm.world >= 4):
        prod = _channel_products(rows_op, cols_op, n, comm, incoming, stream)
        del planes, rows_op, cols_op
        _trimul_out(module, prod, xn, x, n, n_loc, n_pad, stream)
        return
    prod = torch.empty(128, n_loc, n_pad, device=x.device, dtype=_BF16)
    plane = n_loc * n_pad
    # The other ranks' column planes arrive in channel groups: the per-channel
    # products of group g run while group g + 1 is still being gathered.
    groups = 4 if comm.world > 1 else 1
    cg = 128 // groups
    pending = [comm.all_gather_async(cols_op[g * cg:(g + 1) * cg]) for g in range(groups)]
    for g in range(groups):
        cols_all = pending[g].wait()  # [P, cg, n_loc, n_pad]
        off = g * cg * plane * 2
        for p in range(comm.world):
            # O_c[i in I_r, j in I_p] = sum_k rows_c[i, k] cols_c[p][j, k]
            call("bl_batched_gemm", rows_op.data_ptr() + off, 0, n_pad, plane, cols_all[p].data_ptr(), 0, n_pad,
                 plane, prod.data_ptr() + off + p * n_loc * 2, n_pad, plane, cg, n_loc, n_loc, n, None, stream)
        del cols_all
    _trimul_out(module, prod, xn, x, n, n_loc, n_pad, stream)


def _trimul_out(module, prod, xn, x, n, n_loc, n_pad, stream):
    """LayerNorm over the product planes, p_out, g_out(x_hat), gate, z_slab += ."""
    w = forwards._multiplication_weights(module)
    norm = module.norm_out
    call("bl_trimul_output", prod.data_ptr(), n, n_loc, n_pad, _f32(norm.weight).data_ptr(),
         _f32(norm.bias).data_ptr(), float(norm.eps), xn.data_ptr(), w["w_pg"].data_ptr(), x.data_ptr(), None,
         stream)


def _attention_slab(module, x, mask_rows, comm):
    """z_slab += starting-node triangle attention of `module` on the row slab x."""
    n_loc, n = x.shape[0], x.shape[1]
    n_pad = forwards._pad8(n)
    w = forwards._attention_weights(module)
    stream = stream_of(x)
    ln = module.layer_norm
    proj = torch.empty(n_loc * n, 512, device=x.device, dtype=_BF16)
    bias = torch.empty(4, n_loc, n_pad, device=x.device, dtype=_BF16)
    call("bl_attention_projection", x.data_ptr(), n, n_loc, _f32(ln.weight).data_ptr(), _f32(ln.bias).data_ptr(),
         float(ln.eps), w["w_in"].data_ptr(), w["b_in"].data_ptr(), _Q_SCALE, w["w_heads"].data_ptr(), 0,
         proj.data_ptr(), 512, bias.data_ptr(), n_pad, n_loc * n_pad, stream)
    bias_full = _gather_rows(bias, comm).contiguous()  # [4, N, n_pad]
    gated = torch.empty(n_loc * n, 128, device=x.device, dtype=_BF16)
    base = proj.data_ptr()
    call("bl_triangle_attention_residual", base, base + 128 * 2, base + 256 * 2, base + 384 * 2, 512, n, 1,
         bias_full.data_ptr(), n_pad, n * n_pad, mask_rows.data_ptr(), n, 1, float(getattr(module, "inf", 1e9)),
         4, 32, n, n_loc, gated.data_ptr(), 128, w["w_out"].data_ptr(), w["b_out"].data_ptr(), x.data_ptr(), 128,
         stream)


class ShardedPairformer:
    """One Pairformer block (`layers.PairformerLayer` weights) on a row slab.

    forward(s, z_rows, mask, pair_mask) -> (s, z_rows): s [1, N, c_s] and the
    masks are replicated; z_rows [n_loc, N, 128] fp32 holds this rank's rows
    (rank r: rows r * n_loc ...) and the returned slab holds the updated rows
    (the input slab is used as scratch).  N must be a multiple of 8 * world."""

    def __init__(self, block, comm):
        self.block, self.comm = block, comm

    def forward(self, s, z_rows, mask, pair_mask):
        comm, blk = self.comm, self.block
        n_loc, n = z_rows.shape[0], z_rows.shape[1]
        if n % (8 * comm.world) or n_loc * comm.world != n:
            raise RuntimeError("row sharding needs N divisible by 8 * world and equal slabs")
        r0 = comm.rank * n_loc
        pm = pair_mask.reshape(n, n).float()
        mask_rows = pm[r0:r0 + n_loc].contiguous()
        mask_cols = pm.t()[r0:r0 + n_loc].contiguous()
        _trimul_slab(blk.tri_mul_out, z_rows, mask_rows, comm, swap=False)
        if _channel_split(comm) or comm.world == 1:
            # The channel split makes the incoming contraction (over rows) local.
            _trimul_slab(blk.tri_mul_in, z_rows, mask_rows, comm, swap=False, incoming=True)
        else:
            z_cols = rows_to_columns(z_rows, comm)
            _trimul_slab(blk.tri_mul_in, z_cols, mask_cols, comm, swap=True)
            z_rows = rows_to_columns(z_cols, comm)
        _attention_slab(blk.tri_att_start, z_rows, mask_rows, comm)
        z_cols = rows_to_columns(z_rows, comm)
        _attention_slab(blk.tri_att_end, z_cols, mask_cols, comm)
        z_rows = rows_to_columns(z_cols, comm)
        forwards.transition_forward(blk.transition_z, z_rows, residual=z_rows)
        s = self._single_track(s, z_rows, mask)
        return s, z_rows

    __call__ = forward

    def _single_track(self, s, z_rows, mask):
        """s += AttentionPairBias(LN(s), z); s += Transition(s), sharded by query rows.

        Rank r holds z rows I_r, so the pair bias rows bias[h, i, :] for its own queries
        i in I_r are local (bl_pair_bias on the slab).  LN(s) and the q | k | v | g
        projection run for all tokens (replicated; small next to the pair ops), the
        attention of the n_loc local queries against all N keys reads q / g at the local
        rows (bl_token_attention with n_q = n_loc), proj_o adds the residual s[I_r], and
        transition_s runs on the local rows.  One all_gather of the updated s rows
        (N x c_s fp32) then gives every rank the full s: the [H, N, N] fp32 bias is never
        gathered and the attention is not replicated."""
        blk, comm = self.block, self.comm
        att = blk.attention
        n_loc, n = z_rows.shape[0], z_rows.shape[1]
        r0 = comm.rank * n_loc
        heads, d = att.num_heads, att.head_dim
        s = s.contiguous()
        c = s.shape[-1]
        if (d not in forwards._TOKEN_HEAD_DIMS or heads * d != c or s.dtype != torch.float32 or c % 128 or c > 1024
                or any(lyr.bias is not None for lyr in (att.proj_k, att.proj_v, att.proj_g))):
            raise RuntimeError("the sharded single track needs fp32 s [1, N, H*d] with d in (24, 32, 48, 64)")
        ln, lin = att.proj_z[0], att.proj_z[1]
        w_z = lin.weight.float().contiguous()
        stream = stream_of(z_rows)
        bias_loc = torch.empty(1, heads, n_loc, n, device=z_rows.device, dtype=torch.float32)
        call("bl_pair_bias", z_rows.data_ptr(), n_loc * n, _lib.ptr(ln.weight), _lib.ptr(ln.bias), float(ln.eps),
             w_z.data_ptr(), heads, bias_loc.data_ptr(), stream)
        s3 = kernels.layer_norm_split3(s, blk.pre_norm_s.weight, blk.pre_norm_s.bias, blk.pre_norm_s.eps)
        proj = forwards._linear32_planes(att, "_bl_w3_qkvg", s3, (1, n),
                                         [att.proj_q.weight, att.proj_k.weight, att.proj_v.weight, att.proj_g.weight],
                                         [att.proj_q.bias, None, None, None])  # [1, N, 4c]: q | k | v | g
        base, row = proj.data_ptr(), 4 * c * 4
        out3 = torch.empty(3, n_loc, c, device=s.device, dtype=torch.bfloat16)
        maskf = None if mask is None else mask.float().contiguous()
        kernels.launch_token_attention(base + r0 * row, base + c * 4, base + 2 * c * 4, base + r0 * row + 3 * c * 4,
                                       (n * 4 * c, 4 * c, d), bias_loc, maskf, att.inf, 1, heads, n, d, None,
                                       stream, out3=out3, n_q=n_loc)
        s_loc = forwards._linear32_planes(att, "_bl_w3_o", out3, (n_loc,), [att.proj_o.weight], [att.proj_o.bias],
                                          residual=s[0, r0:r0 + n_loc].contiguous())
        s_loc = blk.transition_s(s_loc, residual=s_loc)
        return comm.all_gather(s_loc).reshape(1, n, c)
