"""Tensor-parallel int4 projections (one process per GPU, torch.distributed over NCCL).

Column-parallel matrices (q/k/v, gate/up) keep a contiguous block of output rows per rank; row-
parallel matrices (o, down) keep a contiguous block of the K axis per rank, cut on 32-group
boundaries so every rank's scales stay whole, and their partial outputs are summed across ranks
(all-reduce, fp32). The reference has no multi-device path; the split follows the usual Megatron
layout for a decoder layer: q/k/v and gate/up by output rows (heads), o and down by input columns.

Weights are int4 packed along K (uint8 [N, K/2], element 2j in the low nibble of byte j) with fp16
scales [N, K/32], the layout `DenseMatrix.from_int4` takes.
"""
import torch

from .dense import DenseMatrix, EPI_BF16, EPI_F32, EPI_SWIGLU, EPI_SWIGLU_F32

GROUP = 32


def split_range(n, rank, world, align=1):
    """[lo, hi) of rank's block when n items are split evenly in units of `align`."""
    if n % (world * align):
        raise ValueError(f"{n} does not split into {world} blocks of a multiple of {align}")
    b = n // world
    return rank * b, (rank + 1) * b


def column_shard(qk, s, rank, world):
    """Output rows [lo, hi) of an [N, K] int4 matrix."""
    lo, hi = split_range(qk.shape[0], rank, world)
    return qk[lo:hi], s[lo:hi]


def row_shard(qk, s, rank, world):
    """Input columns [k0, k1) of an [N, K] int4 matrix, K cut on 32-group boundaries."""
    K = qk.shape[1] * 2
    k0, k1 = split_range(K, rank, world, GROUP)
    return qk[:, k0 // 2:k1 // 2], s[:, k0 // GROUP:k1 // GROUP]


def fused_rows_shard(parts, rank, world):
    """Column shard of several matrices stacked by rows (q | k | v, or gate | up): each part
    contributes its own rank block, in order. parts: [(qk, s), ...]."""
    sh = [column_shard(qk, s, rank, world) for qk, s in parts]
    return torch.cat([q for q, _ in sh]), torch.cat([s for _, s in sh])


class TPLinear:
    """One rank's shard of an int4 projection. kind "column": y = x . W_shard^T (a block of the
    output); kind "row": y = sum over ranks of x_shard . W_shard^T, all-reduced by `allreduce`
    (a comm.PeerAllReduce: one launch over NVLink peer memory) or, when only a process group is
    given, by NCCL."""

    def __init__(self, qk, s, kind, gateup=False, group=None, allreduce=None):
        assert kind in ("column", "row")
        self.kind, self.group, self.allreduce = kind, group, allreduce
        self.m = DenseMatrix.from_int4(qk, s, gateup=gateup)
        self.N, self.K = self.m.N, self.m.K

    def __call__(self, x, out, epi=EPI_F32, stream=None, reduce=True, out_bf16=None):
        """out_bf16 (row-parallel): also receive the reduced sum as bf16 (the next projection's
        input). With the peer all-reduce, the GEMV's epilogue sends its outputs to the peers itself
        (onpu_dense_mv_allreduce_dev) and the receiving launch writes both outputs."""
        if self.kind == "row" and reduce and self.allreduce is not None and epi == EPI_F32:
            return self.allreduce.linear(self.m, x, out=out, out_bf16=out_bf16, stream=stream)
        self.m.mv(x, out=out, epi=epi, stream=stream)
        if self.kind == "row" and reduce:
            if self.allreduce is not None:
                self.allreduce(out, out=out, out_bf16=out_bf16, stream=stream)
                return out
            if self.group is not None:
                torch.distributed.all_reduce(out, group=self.group)
        if out_bf16 is not None:
            out_bf16.copy_(out)
        return out


    def mm(self, x, out, epi=EPI_F32, stream=None, reduce=True):
        """Prefill (many rows) on the tensor cores (DenseMatrix.mm, fp16 operands, fp32
        accumulation); a row-parallel shard's partial output is then all-reduced over the group
        (NCCL), as for decode. x: bf16 [M, K_shard or K]."""
        self.m.mm(x, out=out, epi=epi, stream=stream)
        if self.kind == "row" and reduce and self.group is not None:
            if stream is not None:
                with torch.cuda.stream(stream):
                    torch.distributed.all_reduce(out, group=self.group)
            else:
                torch.distributed.all_reduce(out, group=self.group)
        return out


class TPMLP:
    """One rank's shard of a SwiGLU MLP for prefill: gate/up column-parallel (this rank's block of
    gate rows stacked on its block of up rows, so the GEMM's SwiGLU epilogue stays fused), down
    row-parallel (this rank's K block) followed by an all-reduce of the [M, hidden] fp32 output."""

    def __init__(self, gu, dn, group=None):
        self.gu = TPLinear(*gu, "column", gateup=True, group=group)
        self.dn = TPLinear(*dn, "row", group=group)

    @classmethod
    def from_full(cls, gate, up, down, rank, world, group=None):
        return cls(fused_rows_shard([gate, up], rank, world), row_shard(*down, rank, world), group)

    def __call__(self, x, a, y, stream=None, reduce=True):
        """x bf16 [M, hidden]; a bf16 [M, inter / world] (the activation); y fp32 [M, hidden]."""
        self.gu.mm(x, a, epi=EPI_SWIGLU, stream=stream)
        return self.dn.mm(a, y, stream=stream, reduce=reduce)


class TPDecoderLayer:
    """One decoder layer's projections on one rank: q/k/v (column), o (row), gate/up with the
    SwiGLU epilogue (column), down (row). Attention is not part of the path: o takes this rank's
    q-projection output (its heads) as the stand-in for the attention output of those heads.
    The layer's input x ([M, hidden], the same on every rank) and output (fp32 [M, hidden],
    all-reduced) likewise.

    Decode (M up to f32_rows, the most fp32 rows every projection's GEMV keeps in shared memory):
    every activation between the projections stays fp32, as in the reference's
    dequantise-then-matmul path (opennpu/native/reference.py:55-57, :84); each GEMV stages its fp32
    input as two fp16 halves per value. Longer batches carry bf16 activations between the
    projections (the rounding the reference's device path applies to every NPU input)."""

    def __init__(self, qkv, o, gu, dn, nq, group=None, allreduce=None):
        """qkv / gu: this rank's stacked row blocks (q|k|v, gate|up); o / dn: its K blocks; each an
        (int4 codes, fp16 scales) pair. nq: this rank's q rows (= o's K block). allreduce: None
        (NCCL), or a pair of comm.PeerAllReduce, one for o and one for down (a communicator serves
        one call site: the fused GEMV's CTAs sum rows fixed by the shape)."""
        ar_o, ar_dn = allreduce if allreduce is not None else (None, None)
        self.qkv = TPLinear(*qkv, "column", group=group)
        self.o = TPLinear(*o, "row", group=group, allreduce=ar_o)
        self.gu = TPLinear(*gu, "column", gateup=True, group=group)
        self.dn = TPLinear(*dn, "row", group=group, allreduce=ar_dn)
        self.nq = nq
        assert self.o.K == nq
        self.f32_rows = min(p.m.max_f32_rows() for p in (self.qkv, self.o, self.gu, self.dn))

    @classmethod
    def from_full(cls, w, rank, world, group=None, allreduce=None):
        """w: dict of full matrices (codes, scales) for q, k, v, o, gate, up, down."""
        nq = split_range(w["q"][0].shape[0], rank, world)
        return cls(fused_rows_shard([w["q"], w["k"], w["v"]], rank, world), row_shard(*w["o"], rank, world),
                   fused_rows_shard([w["gate"], w["up"]], rank, world), row_shard(*w["down"], rank, world),
                   nq[1] - nq[0], group, allreduce)

    def buffers(self, M, device="cuda"):
        dt = torch.float32 if M <= self.f32_rows else torch.bfloat16
        return {"qkv": torch.empty(M, self.qkv.N, device=device, dtype=dt),
                "h": torch.empty(M, self.o.N, device=device),
                "x2": torch.empty(M, self.o.N, device=device, dtype=torch.bfloat16),
                "a": torch.empty(M, self.gu.N // 2, device=device, dtype=dt),
                "y": torch.empty(M, self.dn.N, device=device)}

    def __call__(self, x, b, stream=None, y_bf16=None):
        """x: [M, hidden] (fp32 or bf16 for M <= 8, else bf16); b: buffers(); returns b["y"] (fp32,
        summed over ranks). y_bf16: also receive the output as bf16 (the next layer's input when
        the activations are bf16)."""
        if b["qkv"].dtype == torch.float32:
            self.qkv(x, b["qkv"], epi=EPI_F32, stream=stream)
            self.o(b["qkv"][:, :self.nq], b["h"], stream=stream)
            self.gu(b["h"], b["a"], epi=EPI_SWIGLU_F32, stream=stream)
        else:
            if x.dtype != torch.bfloat16:           # these rows take the bf16 path (too many for fp32)
                x = x.to(torch.bfloat16)
            self.qkv(x, b["qkv"], epi=EPI_BF16, stream=stream)
            self.o(b["qkv"][:, :self.nq], b["h"], stream=stream, out_bf16=b["x2"])
            self.gu(b["x2"], b["a"], epi=EPI_SWIGLU, stream=stream)
        self.dn(b["a"], b["y"], stream=stream, out_bf16=y_bf16)
        return b["y"]


def dense_layer_shapes(hidden, inter, q_heads, kv_heads, head_dim=128):
    """(name, N, K) of a decoder layer's projections."""
    q, kv = q_heads * head_dim, kv_heads * head_dim
    return [("q", q, hidden), ("k", kv, hidden), ("v", kv, hidden), ("o", hidden, q),
            ("gate", inter, hidden), ("up", inter, hidden), ("down", hidden, inter)]
