"""B200PlanEmitter: LoweredModel -> static launch plan (+ packed weight blob).

This is the new emit target beside the reference's ``CEmitter.emit_model``
(src/emx_onnx_cgen/codegen/c_emitter.py:1312) and ``collect_weight_data``
(:4398).  Instead of rendering one C loop nest per lowered op it decides, for
the same op sequence:

* a kernel per op (or per fused group of ops), in ``LoweredModel.ops`` order;
* a fixed place for every tensor: weights at offsets in one weight blob
  (re-packed into the layouts the kernels read, e.g. conv weights as
  tensor-core operand images), every intermediate at an offset in one device
  arena sized here, so nothing is allocated at run time;
* internal layouts between kernels (zero-bordered NHWC activations between
  tensor-core convolutions) and graph-level fusions (QLinearAdd into the
  epilogue of the convolution that produces one of its operands).

Ops without a B200 kernel raise ``UnsupportedOpError``: there is no CPU
fallback.  The emitter only reads op class names and fields, so it accepts the
reference's own ``LoweredModel`` as well as ``emx_onnx_cgen_b200.lowering``'s.

The binary format is defined in ``csrc/plan_format.h``; kernel ids and
parameter slots in ``csrc/kernels.h`` (mirrored in ``kernel_ids.py``).
"""
from __future__ import annotations

import math
import struct
from dataclasses import dataclass, field

import numpy as np

from . import kernel_ids as K
from .lowering import UnsupportedOpError

PLAN_MAGIC = 0x50584D45
PLAN_VERSION = 1
MAX_RANK = 8
OP_MAX_T, OP_MAX_I, OP_MAX_F = 12, 40, 8
T_WEIGHT, T_INPUT, T_OUTPUT, T_TEMP = 0, 1, 2, 3
DT = {"f32": 1, "u8": 2, "i8": 3, "i32": 6, "i64": 7, "f16": 10, "f64": 11}
NP = {"f32": np.float32, "u8": np.uint8, "i8": np.int8, "i32": np.int32, "i64": np.int64,
      "f16": np.float16, "f64": np.float64}
ALIGN = 256

_HDR = struct.Struct("<IIIIIIqQQII")
_TENSOR = struct.Struct("<IIQQii8q")
_OP = struct.Struct("<II12i40q8d")
assert _HDR.size == 56 and _TENSOR.size == 96 and _OP.size == 440


def _suffix(dt) -> str:
    return str(getattr(dt, "value", dt))


def _name(obj) -> str:
    return type(obj).__name__


def _fn(op) -> str:
    f = getattr(op, "function", None)
    return str(getattr(f, "name", f)).upper()


@dataclass
class PlanTensor:
    kind: int
    dtype: str
    offset: int
    nbytes: int
    shape: tuple[int, ...]
    batch_axis: int = -1
    name: str = ""


@dataclass
class PlanOp:
    kernel: int
    tensors: list[int]
    ip: dict[int, int] = field(default_factory=dict)
    fp: dict[int, float] = field(default_factory=dict)
    label: str = ""


@dataclass
class Plan:
    """A serialisable launch plan: ``plan_bytes`` + ``weight_bytes`` is what
    ``emx_b200_plan_load_mem`` consumes."""
    name: str
    plan_bytes: bytes
    weight_bytes: bytes
    input_names: tuple[str, ...]
    input_shapes: tuple[tuple[int, ...], ...]
    input_dtypes: tuple[str, ...]
    output_names: tuple[str, ...]
    output_shapes: tuple[tuple[int, ...], ...]
    output_dtypes: tuple[str, ...]
    batch: int
    ops: list[PlanOp]
    tensors: list[PlanTensor]
    arena_bytes: int

    def describe(self) -> str:
        lines = [f"plan {self.name}: {len(self.ops)} ops, arena {self.arena_bytes} B, "
                 f"weights {len(self.weight_bytes)} B, batch {self.batch}"]
        for op in self.ops:
            lines.append(f"  {K.NAMES.get(op.kernel, op.kernel):>16}  {op.label}")
        return "\n".join(lines)


class _Builder:
    def __init__(self):
        self.tensors: list[PlanTensor] = []
        self.weights = bytearray()
        self.arena = 0
        self.ops: list[PlanOp] = []
        self.all_batched = True

    def weight(self, arr: np.ndarray, dtype: str, name: str = "") -> int:
        arr = np.ascontiguousarray(arr)
        off = len(self.weights)
        self.weights += arr.tobytes()
        pad = (-len(self.weights)) % ALIGN
        self.weights += b"\0" * pad
        self.tensors.append(PlanTensor(T_WEIGHT, dtype, off, arr.nbytes, tuple(arr.shape), -1, name))
        return len(self.tensors) - 1

    def arena_tensor(self, kind: int, dtype: str, shape, nbytes: int | None = None, batch_axis: int = -1,
                     name: str = "") -> int:
        shape = tuple(int(s) for s in shape)
        if nbytes is None:
            nbytes = int(np.prod(shape, dtype=np.int64)) * np.dtype(NP[dtype]).itemsize
        off = self.arena
        self.arena += (nbytes + ALIGN - 1) // ALIGN * ALIGN
        self.tensors.append(PlanTensor(kind, dtype, off, nbytes, shape, batch_axis, name))
        return len(self.tensors) - 1

    def op(self, kernel: int, tensors, ip=None, fp=None, label="", batched: bool = False) -> None:
        ip = dict(ip or {})
        ip[K.IP_BATCHED_SLOT] = 1 if batched else 0
        self.ops.append(PlanOp(kernel, list(tensors), ip, dict(fp or {}), label))
        if not batched:
            self.all_batched = False

    def serialize(self, inputs: list[int], outputs: list[int], batch: int, flags: int) -> bytes:
        out = bytearray()
        arena = self.arena + ALIGN
        out += _HDR.pack(PLAN_MAGIC, PLAN_VERSION, len(self.tensors), len(self.ops), len(inputs), len(outputs),
                         batch, arena, len(self.weights), flags, 0)
        for t in self.tensors:
            dims = list(t.shape)[:MAX_RANK] + [0] * (MAX_RANK - min(len(t.shape), MAX_RANK))
            out += _TENSOR.pack(t.kind, DT[t.dtype], t.offset, t.nbytes, len(t.shape), t.batch_axis, *dims)
        for ids in (inputs, outputs):
            slots = list(ids) + [0] * (len(ids) % 2)
            out += struct.pack(f"<{len(slots)}I", *slots)
        for op in self.ops:
            t = op.tensors + [-1] * (OP_MAX_T - len(op.tensors))
            ip = [0] * OP_MAX_I
            for k, v in op.ip.items():
                ip[k] = int(v)
            fp = [0.0] * OP_MAX_F
            for k, v in op.fp.items():
                fp[k] = float(v)
            out += _OP.pack(op.kernel, len(op.tensors), *t, *ip, *fp)
        return bytes(out)


def qadd_table(c_signed: bool, c_zero: int, c_scale, r_signed: bool, r_zero: int, r_scale, y_scale, y_zero: int,
               y_signed: bool) -> np.ndarray:
    """QLinearAdd of every (conv byte, residual byte) pair, as the reference
    evaluates it in float (templates/qlinear_add_op.c.j2:2-17):
    clamp(nearbyintf(((float)(a-za)*sa + (float)(b-zb)*sb) / ys + zy)).
    Returns the 65536 output bytes indexed by (conv byte << 8) | residual byte."""
    byte = np.arange(256, dtype=np.int64)
    a = (byte.astype(np.uint8).view(np.int8) if c_signed else byte).astype(np.int64)
    b = (byte.astype(np.uint8).view(np.int8) if r_signed else byte).astype(np.int64)
    f32 = np.float32
    ar = (a - c_zero).astype(f32) * f32(c_scale)
    br = (b - r_zero).astype(f32) * f32(r_scale)
    s = ((ar[:, None] + br[None, :]).astype(f32) / f32(y_scale)).astype(f32) + f32(y_zero)
    r = np.clip(np.rint(s.astype(f32)), -128 if y_signed else 0, 127 if y_signed else 255).astype(np.int64)
    return (r & 0xFF).astype(np.uint8).reshape(-1)


def qsoftmax_exp_table(x_signed: bool, x_zero: int, x_scale) -> np.ndarray:
    """[256][256] f32: expf(v(b) - v(bm)) for raw bytes b, bm, where v(q) =
    (float)(q - zx) * xs.  Evaluated once with the C library's expf -- the
    function the reference's generated C calls (templates/qlinear_softmax_op.c.j2)
    -- so the kernel's exp values are the reference's bit for bit; a device
    exp is correctly rounded and differs from glibc's expf in about 1e-4 of
    arguments."""
    import ctypes
    import ctypes.util
    libm = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
    expf = libm.expf
    expf.restype, expf.argtypes = ctypes.c_float, [ctypes.c_float]
    q = np.arange(256, dtype=np.int32)
    if x_signed:
        q = q.astype(np.uint8).view(np.int8).astype(np.int32)
    v = (q - np.int32(x_zero)).astype(np.float32) * np.float32(x_scale)
    args = (v[:, None] - v[None, :]).astype(np.float32)
    uniq, inv = np.unique(args.view(np.uint32), return_inverse=True)
    vals = np.array([expf(float(a)) for a in uniq.view(np.float32)], dtype=np.float32)
    return vals[inv].reshape(256, 256)


def swizzle_positions(rows: int, row_bytes: int) -> np.ndarray:
    """[rows, row_bytes // 16]: position of 16-byte chunk j of row r in the
    tensor-core K-major swizzle of a row_bytes-wide row (same rule as
    swz_chunk in csrc/tc100.cuh)."""
    nchunk = row_bytes // 16
    phase = ((np.arange(rows, dtype=np.int64) * row_bytes) >> 7) & (nchunk - 1)
    return np.arange(nchunk)[None, :] ^ phase[:, None]


def qconv_weight_image(w: np.ndarray) -> np.ndarray:
    """OIHW int8 weights -> the tensor-core operand image [tap][oc][cin]
    (tap = kh*KW + kw), each oc row of cin bytes with its 16-byte chunks in
    swizzled positions."""
    oc, cin, kh, kw = w.shape
    base = np.ascontiguousarray(w.transpose(2, 3, 0, 1)).reshape(kh * kw, oc, cin // 16, 16)
    pos = swizzle_positions(oc, cin)
    img = np.empty_like(base)
    img[:, np.arange(oc)[:, None], pos, :] = base
    return np.ascontiguousarray(img.reshape(kh * kw, oc, cin))


NB_TILE_N, NB_KSTEP = 128, 64
# nibble position p of a packed word holds the word's k offset _NB_PERM[p]:
# (word >> 4i) & 0x000F000F then yields the pair (k = 2i, k = 2i + 1)
_NB_PERM = np.array([0, 2, 4, 6, 1, 3, 5, 7])


def unpack_nbits(b: np.ndarray, n: int, block: int) -> np.ndarray:
    """MatMulNBits B [N][n_blocks][block/2] (4-bit, low nibble first, as
    templates/matmul_nbits_op.c.j2 reads it) -> q [N][n_blocks * block]."""
    nb = np.asarray(b, dtype=np.uint8).reshape(n, -1, block // 2)
    return np.stack([nb & 15, nb >> 4], axis=-1).reshape(n, -1)


def unpack_nbits_zero_points(zp, n: int, n_blocks: int) -> np.ndarray:
    """MatMulNBits zero points -> [N][n_blocks] (lowering/matmul_nbits.py:171-185,
    templates/matmul_nbits_op.c.j2): None -> 8; uint8 of rank >= 2 -> packed
    4-bit per block (block b in byte b/2, low nibble first); rank 1 -> one per
    column (its low nibble)."""
    if zp is None:
        return np.full((n, n_blocks), 8, np.uint8)
    z = np.asarray(zp, dtype=np.uint8)
    if z.ndim < 2:
        return np.repeat((z.reshape(n, 1) & 15), n_blocks, axis=1)
    z = z.reshape(n, -1)
    return np.stack([z & 15, z >> 4], axis=-1).reshape(n, -1)[:, :n_blocks]


def lstm_persistent_fits(b: int, isz: int, h: int, sms: int) -> bool:
    """The persistent LSTM kernel's launch-shape rule (lstm.cu lp_config): one
    CTA per SM holds ceil(H / sms) units' W and R rows and a LP_STAGES-deep
    ring of LP_KC activation columns for every batch row (at most 256 rows,
    one TMA box), with one compute warp per 32 x RB rows of a unit plus a
    producer warp."""
    rb = 4 if b > 64 else (2 if b > 32 else 1)
    wu = -(-b // (32 * rb))
    bpad = wu * 32 * rb
    u = -(-h // sms)
    grid = -(-h // u)
    threads = u * wu * 32 + 32
    smem = 1024 + u * 4 * (isz + h) * 4 + K.LP_STAGES * bpad * K.LP_KC * 4 + (2 * K.LP_STAGES + 1) * 8
    return (isz % K.LP_KC == 0 and h % K.LP_KC == 0 and bpad <= 256 and threads <= K.LP_MAX_THREADS
            and smem <= K.LP_SMEM_LIMIT and grid <= sms)


def qconv_int_requant_ok(w: np.ndarray, bias: np.ndarray, scale: np.ndarray, a_signed: int) -> int:
    """1 when every accumulator the weights allow keeps |(float)acc * scale| < 2^21.

    acc = bias + sum (x - zx) * w with |x - zx| <= 128 (int8 operands) or 255
    (raw uint8 with zero point 0).  Below 2^21 (well inside 2^22) the kernel's
    rint by adding 1.5 * 2^23 is exact and the result plus the zero point fits
    an int32, so rounding, zero point and the clamp to the output range run as
    one integer saturating pack with the reference's result
    (qlinear_conv_op.c.j2:34-38)."""
    if not np.all(np.isfinite(scale)):
        return 0
    oc = w.shape[0]
    xmax = 128 if a_signed else 255
    acc = xmax * np.abs(w.astype(np.int64)).reshape(oc, -1).sum(1) + np.abs(bias.astype(np.int64))
    return int(float((acc.astype(np.float64) * np.abs(scale.astype(np.float64))).max()) < 2.0 ** 21)


def nbits_weight_image(parts, k: int, block: int, fused: bool):
    """Weight image of the tcgen05 MatMulNBits kernel.

    ``parts`` is [(q [N][Kq] uint8, zp [N][n_blocks] uint8, scales [N][n_blocks]
    fp16, bias [N] f32 | None)] - one entry, or (gate, up) when ``fused``.
    Tile rows: plain, 128 consecutive columns; fused, 64 gate columns then the
    same 64 up columns.  Per (tile, K step of 64) one block of
    4096 + 512 * G bytes: packed words [2][128][4] (see _NB_PERM) then
    [128][G] words (scale fp16 | -(1024 + zp) fp16 << 16), G = 64 / SG scale
    groups of SG = min(block, 32) columns.  Padding rows and columns dequantise
    to exactly 0.  Returns (image bytes, bias f32 [n_tiles*128] | None,
    n_tiles, k_steps, G)."""
    n = parts[0][0].shape[0]
    n_blocks = parts[0][1].shape[1]
    sg = 32 if block >= 32 else 16
    groups = NB_KSTEP // sg
    k_steps = -(-k // NB_KSTEP)
    kp = k_steps * NB_KSTEP
    half = NB_TILE_N // 2 if fused else NB_TILE_N
    n_tiles = -(-n // half)
    rows = n_tiles * NB_TILE_N
    # source (part, column) of every tile row; -1 = padding
    src_col = np.full(rows, -1, np.int64)
    src_part = np.zeros(rows, np.int64)
    t = np.arange(rows)
    tile, r = t // NB_TILE_N, t % NB_TILE_N
    if fused:
        col = tile * half + (r % half)
        src_part = (r >= half).astype(np.int64)
    else:
        col = tile * half + r
    src_col = np.where(col < n, col, -1)

    q = np.full((rows, kp), 8, np.uint8)
    gscale = np.zeros((rows, kp // sg), np.float16)
    gzp = np.full((rows, kp // sg), 8, np.uint8)
    gblk = np.minimum(np.arange(kp // sg) * sg // block, n_blocks - 1)
    gvalid = np.arange(kp // sg) * sg < n_blocks * block
    bias = np.zeros(rows, np.float32)
    have_bias = False
    for pi, (pq, pz, ps, pb) in enumerate(parts):
        sel = (src_part == pi) & (src_col >= 0)
        cols = src_col[sel]
        kk = min(pq.shape[1], kp)
        q[sel, :kk] = pq[cols, :kk]
        gscale[sel] = np.where(gvalid[None, :], ps[cols][:, gblk], np.float16(0))
        gzp[sel] = np.where(gvalid[None, :], pz[cols][:, gblk], 8)
        if pb is not None:
            have_bias = True
            bias[sel] = np.asarray(pb, np.float32)[cols]
    # padded K columns of real rows: q = zp, so the value is exactly 0 whatever the scale
    if kp > n_blocks * block:
        pad_zp = np.repeat(gzp, sg, axis=1)
        q[:, n_blocks * block:] = pad_zp[:, n_blocks * block:]
    words = np.zeros((rows, k_steps, 8), np.uint32)
    qw = q.reshape(rows, k_steps, 8, 8).astype(np.uint32)
    for p_, tk in enumerate(_NB_PERM):
        words |= qw[..., tk] << np.uint32(4 * p_)
    packed = words.reshape(n_tiles, NB_TILE_N, k_steps, 2, 4).transpose(0, 2, 3, 1, 4)
    nbias = (-(1024.0 + gzp.astype(np.float32))).astype(np.float16)
    sw = gscale.view(np.uint16).astype(np.uint32) | (nbias.view(np.uint16).astype(np.uint32) << np.uint32(16))
    sw = sw.reshape(n_tiles, NB_TILE_N, k_steps, groups).transpose(0, 2, 1, 3)
    img = np.concatenate([np.ascontiguousarray(packed).reshape(n_tiles, k_steps, -1).view(np.uint8),
                          np.ascontiguousarray(sw).reshape(n_tiles, k_steps, -1).view(np.uint8)], axis=2)
    return np.ascontiguousarray(img), (bias if have_bias else None), n_tiles, k_steps, groups


def nbits_dequant_from_image(img: np.ndarray, n_tiles: int, k_steps: int, groups: int) -> np.ndarray:
    """Decode a weight image the way the kernel's dequant warps do (fp16
    arithmetic: (1024+q) + -(1024+zp), then x scale, each rounded to fp16) ->
    [n_tiles*128][k_steps*64] fp16, tile row order.  Test helper."""
    stage = img.reshape(n_tiles, k_steps, -1)
    packed = stage[:, :, :4096].copy().view(np.uint32).reshape(n_tiles, k_steps, 2, NB_TILE_N, 4)
    words = packed.transpose(0, 3, 1, 2, 4).reshape(n_tiles * NB_TILE_N, k_steps, 8)
    sw = stage[:, :, 4096:].copy().view(np.uint32).reshape(n_tiles, k_steps, NB_TILE_N, groups)
    sw = sw.transpose(0, 2, 1, 3).reshape(n_tiles * NB_TILE_N, k_steps, groups)
    scale = (sw & 0xFFFF).astype(np.uint16).view(np.float16)
    nb = (sw >> 16).astype(np.uint16).view(np.float16)
    out = np.zeros((n_tiles * NB_TILE_N, k_steps, 8, 8), np.float16)
    for p_, tk in enumerate(_NB_PERM):
        qv = ((words >> np.uint32(4 * p_)) & 15).astype(np.float16) + np.float16(1024)
        g = np.arange(8) * 8 * groups // NB_KSTEP  # chunk j -> its scale group
        out[..., tk] = ((qv + nb[:, :, g]).astype(np.float16) * scale[:, :, g]).astype(np.float16)
    return out.reshape(n_tiles * NB_TILE_N, k_steps * NB_KSTEP)


@dataclass
class _Padded:
    tid: int
    hp: int
    wp: int
    pt: int
    pl: int
    xor: int
    rows: int


class B200PlanEmitter:
    """Emit target producing a B200 launch plan from a LoweredModel."""

    def __init__(self, *, use_tensor_cores: bool = True, nbits_rounded_dequant: bool = False,
                 chain_convs: bool = True, attention_mode: str = "exact"):
        """``nbits_rounded_dequant``: MatMulNBits multiplies fp16-rounded
        dequantised weights (one MMA per K slice, about 2x the throughput)
        instead of the exact hi + lo split; outputs then differ from the
        reference by up to ~2^-12 of sum_k |a_k * deq_k| rather than by
        summation order only.  ``chain_convs``: consecutive tensor-core
        convolutions of one geometry run as one persistent launch (outputs
        are identical either way).  ``attention_mode``: "exact" repeats the
        reference's fp16 statement rounding bit for bit on CUDA cores;
        "tensor" runs fp16 Attention with 128-wide heads on the tensor cores
        (fp32 accumulation and online softmax: closer to the exact value than
        the reference, not bit-identical to it); other head sizes keep the
        exact kernel."""
        if attention_mode not in ("exact", "tensor"):
            raise ValueError(f"attention_mode {attention_mode!r}: 'exact' or 'tensor'")
        self.attention_mode = attention_mode
        self.use_tensor_cores = use_tensor_cores
        self.nbits_rounded_dequant = nbits_rounded_dequant
        self.chain_convs = chain_convs

    # ------------------------------------------------------------------ entry
    def emit_plan(self, model) -> Plan:
        ctx = model.op_context
        self._consts = {c.name: np.asarray(c.data, dtype=NP[_suffix(c.dtype)]).reshape(c.shape)
                        for c in model.constants}
        self._shape = ctx.shape
        self._dtype = lambda n: _suffix(ctx.dtype(n))
        b = _Builder()
        self._b = b
        ops = list(model.ops)
        in_names = tuple(model.input_names)
        out_names = tuple(model.output_names)
        in_shapes = tuple(tuple(s) for s in model.input_shapes)
        out_shapes = tuple(tuple(s) for s in model.output_shapes)

        # batch: common axis-0 extent of every I/O tensor, else not sliceable
        dims0 = {s[0] for s in (*in_shapes, *out_shapes) if len(s) > 0}
        batch = dims0.pop() if len(dims0) == 1 else 0
        flags = 1 if batch > 0 else 0

        self._nchw: dict[str, int] = {}
        self._padded: dict[str, _Padded] = {}
        for name, shp in zip(in_names, in_shapes):
            self._nchw[name] = b.arena_tensor(T_INPUT, self._dtype(name), shp, batch_axis=0 if batch else -1,
                                              name=name)
        self._outputs = {}
        for name, shp in zip(out_names, out_shapes):
            self._outputs[name] = b.arena_tensor(T_OUTPUT, self._dtype(name), shp,
                                                 batch_axis=0 if batch else -1, name=name)
        self._graph_outputs = set(out_names)
        self._batch = batch

        self._analyse(ops)
        for i, op in enumerate(ops):
            outs = self._op_outputs(op)
            if outs and all(int(np.prod(self._shape(o), dtype=np.int64)) == 0 for o in outs):
                # every output is empty (a zero extent): the reference's loops run
                # zero times, so the op launches nothing; its outputs still exist
                for o in outs:
                    if o not in self._nchw:
                        self._dest(o, self._dtype(o), tuple(self._shape(o)))
                continue
            empty_in = [n for n in self._op_inputs(op) if int(np.prod(self._shape(n), dtype=np.int64)) == 0]
            if empty_in:
                # e.g. an LSTM over zero steps or a Gemm with K = 0: outputs that are not
                # sums over the empty extent have no kernel path here
                raise UnsupportedOpError(f"{_name(op)}: empty input {empty_in[0]} with non-empty outputs")
            if i in self._absorbed:
                continue
            handler = getattr(self, "_emit_" + _name(op), None)
            if handler is None:
                raise UnsupportedOpError(f"{_name(op)} has no B200 kernel")
            handler(i, op)
        for name in out_names:
            if name not in self._written_outputs:
                raise UnsupportedOpError(f"graph output {name} is not produced by any op")
        if self.chain_convs:
            self._mark_qconv_chains()
        if batch > 0 and not b.all_batched:
            # some op's leading extent is not the batch: the plan runs whole only
            batch, flags = 0, 0
            for t in b.tensors:
                t.batch_axis = -1
            for op in b.ops:
                op.ip[K.IP_BATCHED_SLOT] = 0

        blob = b.serialize([self._nchw[n] for n in in_names], [self._outputs[n] for n in out_names], batch,
                           flags)
        return Plan(model.name, blob, bytes(b.weights), in_names, in_shapes,
                    tuple(_suffix(d) for d in model.input_dtypes), out_names, out_shapes,
                    tuple(_suffix(d) for d in model.output_dtypes), batch, b.ops, b.tensors, b.arena + ALIGN)

    # ------------------------------------------------------------------ helpers
    def _const(self, name: str | None, what: str) -> np.ndarray:
        if name is None:
            raise UnsupportedOpError(f"{what} missing")
        if name not in self._consts:
            raise UnsupportedOpError(f"{what} '{name}' must be an initializer for the B200 plan")
        return self._consts[name]

    def _scalar(self, name, what):
        arr = self._const(name, what)
        if arr.size != 1:
            raise UnsupportedOpError(f"{what} must be a scalar")
        return arr.reshape(-1)[0]

    def _dest(self, name: str, dtype: str, shape) -> int:
        """Tensor id an op should write ``name`` to (graph output or new temp)."""
        if name in self._graph_outputs:
            self._written_outputs.add(name)
            tid = self._outputs[name]
        else:
            tid = self._b.arena_tensor(T_TEMP, dtype, shape, name=name)
        self._nchw[name] = tid
        return tid

    def _src(self, name: str) -> int:
        if name in self._nchw:
            return self._nchw[name]
        if name in self._consts:
            arr = self._consts[name]
            tid = self._b.weight(arr, self._dtype(name), name)
            self._nchw[name] = tid
            return tid
        raise UnsupportedOpError(f"tensor {name} is not available in row-major layout")

    # ------------------------------------------------------------------ analysis
    def _analyse(self, ops) -> None:
        self._written_outputs: set[str] = set()
        self._absorbed: set[int] = set()
        self._fused_add: dict[int, int] = {}
        producers: dict[str, int] = {}
        consumers: dict[str, list[int]] = {}
        for i, op in enumerate(ops):
            for nm in self._op_outputs(op):
                producers[nm] = i
            for nm in self._op_inputs(op):
                consumers.setdefault(nm, []).append(i)
        self._producers, self._consumers = producers, consumers

        # tensor-core eligible convolutions and the activation storage they need
        self._tc: dict[int, dict] = {}
        for i, op in enumerate(ops):
            if _name(op) == "QLinearConvOp":
                cfg = self._qconv_tc_config(op)
                if cfg is not None:
                    self._tc[i] = cfg
        # fuse QLinearAdd into a tensor-core conv producing one operand
        for j, op in enumerate(ops):
            if _name(op) != "QLinearAddOp":
                continue
            if tuple(op.input0_shape) != tuple(op.input1_shape):
                continue
            for side, other in ((op.input0, op.input1), (op.input1, op.input0)):
                i = producers.get(side)
                if i is None or i not in self._tc or i in self._fused_add:
                    continue
                if len(consumers.get(side, [])) != 1 or side in self._graph_outputs:
                    continue
                if self._dtype(other) not in ("u8", "i8") or self._dtype(op.output) not in ("u8", "i8"):
                    continue
                self._fused_add[i] = j
                self._absorbed.add(j)
                break
        # padded-storage requirements (xor, pads) per tensor from tensor-core consumers
        self._need_pad: dict[str, tuple[int, int, int, int]] = {}  # name -> (pt, pl, pb, pr) + xor
        self._need_xor: dict[str, int] = {}
        changed = True
        while changed:
            changed = False
            self._need_pad.clear()
            self._need_xor.clear()
            for i, cfg in list(self._tc.items()):
                op = ops[i]
                name = op.input0
                pads = cfg["pads"]
                if name in self._need_pad and (self._need_pad[name] != pads or self._need_xor[name] != cfg["xor"]):
                    del self._tc[i]
                    self._fused_add.pop(i, None)
                    changed = True
                    break
                self._need_pad[name] = pads
                self._need_xor[name] = cfg["xor"]
        self._absorbed = set(self._fused_add.values())
        # gate/up MatMulNBits pair + Swish(gate) * up -> one kernel with a fused epilogue
        self._nbits_fused: dict[int, dict] = {}
        for mi, op in enumerate(ops):
            if _name(op) != "BinaryOp" or _fn(op) != "MUL" or self._dtype(op.output) != "f16":
                continue
            for s_name, u_name in ((op.input0, op.input1), (op.input1, op.input0)):
                i_s, i_u = producers.get(s_name), producers.get(u_name)
                if i_s is None or i_u is None:
                    continue
                sw = ops[i_s]
                if _name(sw) != "UnaryOp" or _fn(sw) != "SWISH":
                    continue
                i_g = producers.get(sw.input0)
                if i_g is None or i_g == i_u:
                    continue
                g, u = ops[i_g], ops[i_u]
                if _name(g) != "MatMulNBitsOp" or _name(u) != "MatMulNBitsOp":
                    continue
                if (g.input0 != u.input0 or int(g.k) != int(u.k) or int(g.n) != int(u.n)
                        or int(g.block_size) != int(u.block_size)):
                    continue
                if self._nbits_reject(g) or self._nbits_reject(u):
                    continue
                inter = (g.output, u.output, s_name)
                if any(nm in self._graph_outputs or len(consumers.get(nm, [])) != 1 for nm in inter):
                    continue
                first = min(i_g, i_u)
                if first in self._nbits_fused or any(x in self._absorbed for x in (i_g, i_u, i_s, mi)):
                    continue
                # `const _Float16 alpha = <literal>;` in the reference's helper: fp16-rounded
                alpha = float(np.float16(float(sw.params[0]) if getattr(sw, "params", ()) else 1.0))
                self._nbits_fused[first] = {"gate": g, "up": u, "mul": op, "alpha": alpha}
                self._absorbed.update({max(i_g, i_u), i_s, mi})
                break
        for i, j in self._fused_add.items():
            add = ops[j]
            conv_out = ops[i].output
            resid = add.input1 if add.input0 == conv_out else add.input0
            if resid not in self._need_pad:
                self._need_pad[resid] = (0, 0, 0, 0)
                self._need_xor[resid] = 0
        # which produced tensors must (also) exist row-major
        self._need_rowmajor: set[str] = set(self._graph_outputs)
        tc_inputs = {ops[i].input0 for i in self._tc}
        resid_inputs = set()
        for i, j in self._fused_add.items():
            add = ops[j]
            conv_out = ops[i].output
            resid_inputs.add(add.input1 if add.input0 == conv_out else add.input0)
        for name, cons in consumers.items():
            for c in cons:
                if c in self._absorbed:
                    continue
                if c in self._tc and ops[c].input0 == name:
                    continue
                self._need_rowmajor.add(name)
        self._ops = ops
        # tensors whose axis 0 follows the plan batch
        self._batched_names: set[str] = set()
        if self._batch > 0:
            self._batched_names.update(n for n in self._nchw)  # graph inputs
            for op in ops:
                ins = self._op_inputs(op)
                if not ins or ins[0] not in self._batched_names:
                    continue
                if _name(op) == "GemmOp" and int(op.trans_a):
                    continue
                if _name(op) == "LstmOp":
                    continue
                for o in self._op_outputs(op):
                    shp = tuple(self._shape(o))
                    if shp and shp[0] == self._batch:
                        self._batched_names.add(o)
        del tc_inputs, resid_inputs

    @staticmethod
    def _op_inputs(op):
        fields = {
            "QLinearConvOp": ("input0",), "QLinearAddOp": ("input0", "input1"),
            "GemmOp": ("input_a", "input_b", "input_c"), "UnaryOp": ("input0",), "BinaryOp": ("input0", "input1"),
            "MatMulNBitsOp": ("input0",), "AttentionOp": ("input_q", "input_k", "input_v"),
            "LstmOp": ("input_x",), "QLinearMatMulOp": ("input0", "input1"), "MatMulIntegerOp": ("input0", "input1"),
            "ConvOp": ("input0", "weights", "bias"), "SoftmaxOp": ("input0",), "QuantizeLinearOp": ("input0",),
            "DequantizeLinearOp": ("input0",), "ReshapeOp": ("input0",), "TransposeOp": ("input0",),
            "MaxPoolOp": ("input0",), "QLinearAveragePoolOp": ("input0",), "QLinearSoftmaxOp": ("input0",),
        }.get(_name(op), ())
        return [getattr(op, f) for f in fields if getattr(op, f, None)]

    @staticmethod
    def _op_outputs(op):
        fields = {"LstmOp": ("output_y", "output_y_h", "output_y_c")}.get(_name(op), ("output",))
        return [getattr(op, f) for f in fields if getattr(op, f, None)]

    # ------------------------------------------------------------------ QLinearConv
    TC_VARIANTS = {(32, 32), (32, 64), (64, 32), (64, 64), (64, 128), (128, 64), (128, 128)}

    def _qconv_tc_config(self, op):
        if not self.use_tensor_cores:
            return None
        if op.spatial_rank != 2 or tuple(op.strides) != (1, 1) or tuple(op.dilations) != (1, 1) or op.group != 1:
            return None
        if (op.in_channels, op.out_channels) not in self.TC_VARIANTS:
            return None
        if _suffix(op.weight_dtype) != "i8" or _suffix(op.dtype) not in ("u8", "i8"):
            return None
        try:
            zx = int(self._scalar(op.input_zero_point, "x_zero_point"))
            wz = self._const(op.weight_zero_point, "w_zero_point")
            self._const(op.weight_scale, "w_scale")
            self._scalar(op.input_scale, "x_scale")
            self._scalar(op.output_scale, "y_scale")
            self._scalar(op.output_zero_point, "y_zero_point")
            if op.bias is not None:
                self._const(op.bias, "bias")
        except UnsupportedOpError:
            return None
        if np.any(wz != 0):
            return None
        xdt = _suffix(op.input_dtype)
        if xdt == "u8" and zx == 128:
            xor, a_signed = 0x80, 1
        elif xdt == "u8" and zx == 0:
            xor, a_signed = 0, 0
        elif xdt == "i8" and zx == 0:
            xor, a_signed = 0, 1
        else:
            return None
        kh, kw = op.kernel_shape
        if kh * kw * op.in_channels * op.out_channels > 160 * 1024 or 128 + kw - 1 > 256:
            return None
        pt, pl, pb, pr = op.pads
        return {"xor": xor, "a_signed": a_signed, "pads": (pt, pl, pb, pr)}

    def _padded_of(self, name: str) -> _Padded:
        """Zero-bordered chunk-planar copy of ``name`` (created by a pad op if
        the producer did not write it directly)."""
        if name in self._padded:
            return self._padded[name]
        pd = self._new_padded(name)
        n, c, h, w = self._shape(name)
        src = self._src(name)
        self._b.op(K.K_PAD_NHWC, [src, pd.tid],
                   {K.PAD_N: n, K.PAD_C: c, K.PAD_H: h, K.PAD_W: w, K.PAD_TOP: pd.pt, K.PAD_LEFT: pd.pl,
                    K.PAD_HP: pd.hp, K.PAD_WP: pd.wp, K.PAD_XOR: pd.xor, K.PAD_ROWS: pd.rows},
                   label=f"{name} -> planar", batched=n == self._batch)
        return pd

    def _new_padded(self, name: str) -> _Padded:
        """Allocate the chunk-planar zero-bordered tensor [C/16][rows][16 B];
        rows = N*Hp*Wp + a tail that covers the last conv windows (up to 9
        kernel rows of Wp plus a 256-row window)."""
        pt, pl, pb, pr = self._need_pad[name]
        n, c, h, w = self._shape(name)
        hp, wp = h + pt + pb, w + pl + pr
        rows = n * hp * wp + 9 * wp + 264
        tid = self._b.arena_tensor(T_TEMP, self._dtype(name), (rows, c), name=name + ":swizzled-nhwc")
        pd = _Padded(tid, hp, wp, pt, pl, self._need_xor[name], rows)
        self._padded[name] = pd
        return pd

    def _emit_QLinearConvOp(self, i, op):
        if i in self._tc:
            return self._emit_qconv_tc(i, op, self._tc[i])
        return self._emit_qconv_generic(op)

    def _emit_qconv_generic(self, op):
        if op.spatial_rank != 2:
            raise UnsupportedOpError("QLinearConv: only 2-D convolutions have a B200 kernel")
        xs = np.float32(self._scalar(op.input_scale, "x_scale"))
        ys = np.float32(self._scalar(op.output_scale, "y_scale"))
        zx = int(self._scalar(op.input_zero_point, "x_zero_point"))
        zy = int(self._scalar(op.output_zero_point, "y_zero_point"))
        w = self._const(op.weights, "weights")
        ws = self._const(op.weight_scale, "w_scale").astype(np.float32).reshape(-1)
        wz = self._const(op.weight_zero_point, "w_zero_point").astype(np.int32).reshape(-1)
        t_w = self._b.weight(w, _suffix(op.weight_dtype), op.weights)
        t_ws = self._b.weight(ws, "f32")
        t_wz = self._b.weight(wz, "i32")
        t_b = -1
        if op.bias is not None:
            t_b = self._b.weight(self._const(op.bias, "bias").astype(np.int32), "i32")
        x = self._src(op.input0)
        n, c, h, wd = self._shape(op.input0)
        oh, ow = op.out_spatial
        y = self._dest(op.output, _suffix(op.dtype), (n, op.out_channels, oh, ow))
        kh, kw = op.kernel_shape
        self._b.op(K.K_QCONV_GENERIC, [x, t_w, t_ws, t_wz, t_b, y], {
            K.QG_N: n, K.QG_C: c, K.QG_H: h, K.QG_W: wd, K.QG_OC: op.out_channels, K.QG_KH: kh, K.QG_KW: kw,
            K.QG_OH: oh, K.QG_OW: ow, K.QG_SH: op.strides[0], K.QG_SW: op.strides[1], K.QG_PT: op.pads[0],
            K.QG_PL: op.pads[1], K.QG_DH: op.dilations[0], K.QG_DW: op.dilations[1], K.QG_GROUP: op.group,
            K.QG_X_SIGNED: int(_suffix(op.input_dtype) == "i8"), K.QG_W_SIGNED: int(_suffix(op.weight_dtype) == "i8"),
            K.QG_Y_SIGNED: int(_suffix(op.dtype) == "i8"), K.QG_X_ZERO: zx, K.QG_Y_ZERO: zy,
            K.QG_WS_PER_CH: int(ws.size > 1), K.QG_WZ_PER_CH: int(wz.size > 1)},
            {K.QGF_X_SCALE: float(xs), K.QGF_Y_SCALE: float(ys)}, label=f"{op.output} (generic)",
            batched=n == self._batch)

    def _emit_qconv_tc(self, i, op, cfg):
        xs = np.float32(self._scalar(op.input_scale, "x_scale"))
        ys = np.float32(self._scalar(op.output_scale, "y_scale"))
        zy = int(self._scalar(op.output_zero_point, "y_zero_point"))
        w = self._const(op.weights, "weights").astype(np.int8)
        oc, cin, kh, kw = w.shape
        ws = self._const(op.weight_scale, "w_scale").astype(np.float32).reshape(-1)
        ws = np.broadcast_to(ws, (oc,)).astype(np.float32)
        # per-channel requant scale exactly as the reference's float expression: (xs * ws) / ys
        scale = (np.float32(xs) * ws).astype(np.float32) / np.float32(ys)
        scale = scale.astype(np.float32)
        bias = (self._const(op.bias, "bias").astype(np.int32) if op.bias is not None
                else np.zeros(oc, np.int32))
        epi = np.concatenate([scale.view(np.uint8), bias.view(np.uint8)])
        t_w = self._b.weight(qconv_weight_image(w), "i8", op.weights + ":tc")
        t_e = self._b.weight(epi, "u8", op.weights + ":epi")
        xin = self._padded_of(op.input0)
        n, _, h, wd = self._shape(op.input0)
        oh, ow = op.out_spatial
        ip = {K.QC_N: n, K.QC_CIN: cin, K.QC_OC: oc, K.QC_KH: kh, K.QC_KW: kw, K.QC_HP: xin.hp, K.QC_WP: xin.wp,
              K.QC_OH: oh, K.QC_OW: ow, K.QC_A_SIGNED: cfg["a_signed"], K.QC_Y_ZERO: zy,
              K.QC_Y_SIGNED: int(_suffix(op.dtype) == "i8"), K.QC_X_ROWS: xin.rows,
              K.QC_RQ_INT: qconv_int_requant_ok(w, bias, scale, cfg["a_signed"])}
        fp = {}
        t_r = t_lut = -1
        out_name = op.output
        out_dtype = _suffix(op.dtype)
        label = f"{op.output}"
        if i in self._fused_add:
            add = self._ops[self._fused_add[i]]
            conv_side0 = add.input0 == op.output
            resid = add.input1 if conv_side0 else add.input0
            c_s = add.input0_scale if conv_side0 else add.input1_scale
            c_z = add.input0_zero_point if conv_side0 else add.input1_zero_point
            r_s = add.input1_scale if conv_side0 else add.input0_scale
            r_z = add.input1_zero_point if conv_side0 else add.input0_zero_point
            rp = self._padded_of(resid)
            t_r = rp.tid
            lut = qadd_table(_suffix(op.dtype) == "i8", int(self._scalar(c_z, "add zero")),
                             np.float32(self._scalar(c_s, "add scale")), self._dtype(resid) == "i8",
                             int(self._scalar(r_z, "add zero")), np.float32(self._scalar(r_s, "add scale")),
                             np.float32(self._scalar(add.output_scale, "add scale")),
                             int(self._scalar(add.output_zero_point, "add zero")), _suffix(add.dtype) == "i8")
            t_lut = self._b.weight(lut, "u8", add.output + ":qadd-table")
            ip.update({K.QC_HAS_ADD: 1, K.QC_C_ZERO: int(self._scalar(c_z, "add zero")),
                       K.QC_R_ZERO: int(self._scalar(r_z, "add zero")), K.QC_R_XOR: rp.xor,
                       K.QC_R_SIGNED: int(self._dtype(resid) == "i8"), K.QC_R_HP: rp.hp, K.QC_R_WP: rp.wp,
                       K.QC_R_PT: rp.pt, K.QC_R_PL: rp.pl, K.QC_R_ROWS: rp.rows,
                       K.QC_ADD_ZERO: int(self._scalar(add.output_zero_point, "add zero")),
                       K.QC_ADD_SIGNED: int(_suffix(add.dtype) == "i8")})
            fp = {K.QCF_C_SCALE: float(np.float32(self._scalar(c_s, "add scale"))),
                  K.QCF_R_SCALE: float(np.float32(self._scalar(r_s, "add scale"))),
                  K.QCF_ADD_SCALE: float(np.float32(self._scalar(add.output_scale, "add scale")))}
            out_name = add.output
            out_dtype = _suffix(add.dtype)
            label += f" + {add.output} (fused QLinearAdd)"
        padded_out = out_name in self._need_pad and out_name not in self._need_rowmajor
        if padded_out:
            yp = self._new_padded(out_name)
            ip.update({K.QC_Y_LAYOUT: 0, K.QC_Y_XOR: yp.xor, K.QC_Y_HP: yp.hp, K.QC_Y_WP: yp.wp,
                       K.QC_Y_PT: yp.pt, K.QC_Y_PL: yp.pl, K.QC_Y_ROWS: yp.rows})
            t_y = yp.tid
        else:
            t_y = self._dest(out_name, out_dtype, (n, oc, oh, ow))
            ip.update({K.QC_Y_LAYOUT: 1})
        self._b.op(K.K_QCONV_TC, [xin.tid, t_w, t_e, t_r, t_y, t_lut], ip, fp, label=label + " (tcgen05 i8)",
                   batched=n == self._batch)
        if padded_out is False and out_name in self._need_pad:
            self._padded_of(out_name)  # consumers also need the NHWC copy

    # ------------------------------------------------------------------ conv chains
    QC_MAX_CHAIN = 8
    _QC_GEOMETRY = ("QC_N", "QC_CIN", "QC_OC", "QC_KH", "QC_KW", "QC_HP", "QC_WP", "QC_OH", "QC_OW")

    def _mark_qconv_chains(self):
        """Consecutive tensor-core convolutions where each reads the previous
        one's (swizzled NHWC) output, with one geometry, run as one persistent
        launch: the first op gets QC_CHAIN = length and a zeroed state tensor
        (run epoch, finished CTAs, one progress word per 128-row tile), the
        others QC_CHAIN = -1.  Fused adds in a chain must read a residual in
        the same padded geometry."""
        ops = self._b.ops
        geom = [getattr(K, f) for f in self._QC_GEOMETRY]

        def member_ok(o, head):
            if o.kernel != K.K_QCONV_TC or any(o.ip.get(f) != head.ip.get(f) for f in geom):
                return False
            if o.ip.get(K.IP_BATCHED_SLOT) != head.ip.get(K.IP_BATCHED_SLOT):
                return False
            if o.ip.get(K.QC_HAS_ADD) and (o.ip.get(K.QC_R_HP) != o.ip[K.QC_HP] or o.ip.get(K.QC_R_WP) != o.ip[K.QC_WP]):
                return False
            return True

        i = 0
        while i < len(ops):
            head = ops[i]
            if not member_ok(head, head):
                i += 1
                continue
            j = i
            while (j + 1 < len(ops) and j + 1 - i < self.QC_MAX_CHAIN and member_ok(ops[j + 1], head)
                   and ops[j + 1].tensors[0] == ops[j].tensors[4] and ops[j].ip.get(K.QC_Y_LAYOUT, 0) == 0
                   and ops[j].ip.get(K.QC_Y_HP) == head.ip[K.QC_HP] and ops[j].ip.get(K.QC_Y_WP) == head.ip[K.QC_WP]):
                j += 1
            n_layers = j - i + 1
            if n_layers > 1:
                ip = head.ip
                q_end = (ip[K.QC_N] - 1) * ip[K.QC_HP] * ip[K.QC_WP] + (ip[K.QC_OH] - 1) * ip[K.QC_WP] + ip[K.QC_OW]
                n_tiles = -(-q_end // 128)
                t_state = self._b.arena_tensor(T_TEMP, "u8", (8 * (2 + n_tiles),), name=f"conv-chain{i}:state")
                head.tensors = head.tensors + [-1] * (7 - len(head.tensors))
                head.tensors[6] = t_state
                head.ip[K.QC_CHAIN] = n_layers
                head.label += f" [chain of {n_layers}: one launch]"
                for k in range(i + 1, j + 1):
                    ops[k].ip[K.QC_CHAIN] = -1
                    ops[k].label += " [in chain]"
            i = j + 1

    # ------------------------------------------------------------------ QLinearAdd (standalone)
    def _broadcast_operand(self, name: str, shape, out_shape) -> int:
        """Tensor id of operand ``name`` at the output's shape: the tensor itself,
        or an initializer broadcast once by the planner (a bias row added to
        every batch entry)."""
        if tuple(shape) == tuple(out_shape):
            return self._src(name)
        if name not in self._consts:
            raise UnsupportedOpError("QLinearAdd: only initializer operands may broadcast")
        full = np.ascontiguousarray(np.broadcast_to(self._consts[name].reshape(shape), tuple(out_shape)))
        return self._b.weight(full, self._dtype(name), f"{name}:broadcast")

    def _emit_QLinearAddOp(self, i, op):
        a = self._broadcast_operand(op.input0, op.input0_shape, op.output_shape)
        b_ = self._broadcast_operand(op.input1, op.input1_shape, op.output_shape)
        y = self._dest(op.output, _suffix(op.dtype), op.output_shape)
        count = int(np.prod(op.output_shape))
        batched = self._batch > 0 and len(op.output_shape) > 0 and op.output_shape[0] == self._batch
        self._b.op(K.K_QLINEAR_ADD, [a, b_, y], {
            K.QA_COUNT: count, K.QA_A_SIGNED: int(_suffix(op.input0_dtype) == "i8"),
            K.QA_B_SIGNED: int(_suffix(op.input1_dtype) == "i8"), K.QA_Y_SIGNED: int(_suffix(op.dtype) == "i8"),
            K.QA_A_ZERO: int(self._scalar(op.input0_zero_point, "a_zero")),
            K.QA_B_ZERO: int(self._scalar(op.input1_zero_point, "b_zero")),
            K.QA_Y_ZERO: int(self._scalar(op.output_zero_point, "y_zero")),
            K.QA_BATCH: self._batch if batched else 0},
            {K.QAF_A_SCALE: float(np.float32(self._scalar(op.input0_scale, "a_scale"))),
             K.QAF_B_SCALE: float(np.float32(self._scalar(op.input1_scale, "b_scale"))),
             K.QAF_Y_SCALE: float(np.float32(self._scalar(op.output_scale, "y_scale")))},
            label=op.output, batched=batched)

    # ------------------------------------------------------------------ Gemm (+ Relu)
    def _fused_relu_of(self, i, op):
        """Index of a Relu that only consumes this op's output (fused into its epilogue)."""
        out = op.output
        cons = self._consumers.get(out, [])
        if out in self._graph_outputs or len(cons) != 1:
            return None
        c = self._ops[cons[0]]
        if _name(c) == "UnaryOp" and _fn(c) == "RELU" and c.input0 == out:
            return cons[0]
        return None

    def _emit_GemmOp(self, i, op):
        if self._dtype(op.input_a) != "f32" or self._dtype(op.input_b) != "f32":
            raise UnsupportedOpError("Gemm: only fp32 has a B200 kernel")
        sa, sb = self._shape(op.input_a), self._shape(op.input_b)
        ta, tb = int(op.trans_a), int(op.trans_b)
        m, k = (sa[1], sa[0]) if ta else (sa[0], sa[1])
        n = sb[0] if tb else sb[1]
        a, b_ = self._src(op.input_a), self._src(op.input_b)
        t_c, mode = -1, 0
        if op.input_c is not None:
            cs = tuple(self._shape(op.input_c))
            size = int(np.prod(cs)) if cs else 1
            if size == 1:
                mode = 1
            elif len(cs) == 1:
                mode = 2 if cs[0] == n else 3
            elif cs == (1, n):
                mode = 2
            elif cs == (m, 1):
                mode = 3
            else:
                mode = 4
            t_c = self._src(op.input_c)
        relu_i = self._fused_relu_of(i, op)
        out = op.output
        if relu_i is not None:
            self._absorbed.add(relu_i)
            out = self._ops[relu_i].output
        y = self._dest(out, "f32", (m, n))
        self._b.op(K.K_GEMM_F32, [a, b_, t_c, y], {
            K.GM_M: m, K.GM_N: n, K.GM_K: k, K.GM_TRANS_A: ta, K.GM_TRANS_B: tb, K.GM_BIAS_MODE: mode,
            K.GM_RELU: int(relu_i is not None)},
            {K.GMF_ALPHA: float(np.float32(op.alpha)), K.GMF_BETA: float(np.float32(op.beta))},
            label=f"{op.output}" + (f" + Relu -> {out}" if relu_i is not None else "") + " (fp32, reference order)",
            batched=(not ta) and m == self._batch and self._is_batched(op.input_a))

    def _is_batched(self, name: str) -> bool:
        """Whether tensor ``name``'s axis 0 follows the plan batch (graph input or
        produced from one by batched ops)."""
        return name in self._batched_names

    def _emit_UnaryOp(self, i, op):
        fn = _fn(op)
        dt = self._dtype(op.input0)
        shape = tuple(self._shape(op.input0))
        x = self._src(op.input0)
        y = self._dest(op.output, dt, shape)
        count = int(np.prod(shape))
        rows = shape[0] if shape and shape[0] == self._batch and self._is_batched(op.input0) else 0
        ip = {K.EW_COUNT: count, K.EW_ROWS: rows}
        if fn == "RELU" and dt == "f32":
            self._b.op(K.K_RELU_F32, [x, y], ip, label=op.output, batched=rows > 0)
        elif fn == "SWISH" and dt == "f16":
            alpha = float(np.float16(float(op.params[0]) if getattr(op, "params", ()) else 1.0))
            # 128 KB table of Swish over every fp16 value, filled once at load time
            table = self._b.arena_tensor(T_TEMP, "u8", (2 * 65536,), name=f"{op.output}:swish-table")
            self._b.op(K.K_SWISH_F16, [x, y, table], ip, {K.EWF_ALPHA: alpha}, label=op.output, batched=rows > 0)
        else:
            raise UnsupportedOpError(f"Unary {fn} on {dt} has no B200 kernel")

    def _emit_BinaryOp(self, i, op):
        fn = _fn(op)
        dt = self._dtype(op.output)
        sa, sb = tuple(self._shape(op.input0)), tuple(self._shape(op.input1))
        if fn != "MUL" or dt != "f16" or self._dtype(op.input0) != "f16" or self._dtype(op.input1) != "f16":
            raise UnsupportedOpError(f"Binary {fn} on {dt} has no B200 kernel")
        if sa != sb:
            raise UnsupportedOpError("Mul: broadcasting operands have no B200 kernel")
        a, b_ = self._src(op.input0), self._src(op.input1)
        y = self._dest(op.output, dt, sa)
        rows = (sa[0] if sa and sa[0] == self._batch and self._is_batched(op.input0)
                and self._is_batched(op.input1) else 0)
        self._b.op(K.K_MUL_F16, [a, b_, y], {K.EW_COUNT: int(np.prod(sa)), K.EW_ROWS: rows}, label=op.output,
                   batched=rows > 0)

    # ------------------------------------------------------------------ QLinearMatMul / MatMulInteger
    def _rows_batched(self, name: str, shape) -> tuple[bool, int]:
        """(batched, rows per batch entry) for an op whose rows are shape[:-1]."""
        rows = int(np.prod(shape[:-1])) if len(shape) > 1 else 1
        batched = (self._batch > 0 and len(shape) > 1 and shape[0] == self._batch and self._is_batched(name))
        return batched, (rows // self._batch if batched else 0)

    def _emit_matmul8(self, op, quantized: bool):
        what = "QLinearMatMul" if quantized else "MatMulInteger"
        a_dt, b_dt = self._dtype(op.input0), self._dtype(op.input1)
        if a_dt not in ("u8", "i8") or b_dt not in ("u8", "i8") or len(op.input1_shape) != 2:
            raise UnsupportedOpError(f"{what}: 8-bit A and 2-D 8-bit B only")
        a, b_ = self._src(op.input0), self._src(op.input1)
        batched, rpb = self._rows_batched(op.input0, tuple(op.input0_shape))
        zero = lambda nm, w: 0 if nm is None else int(self._scalar(nm, w))
        ip = {K.QM_M: int(op.m), K.QM_K: int(op.k), K.QM_N: int(op.n), K.QM_A_SIGNED: int(a_dt == "i8"),
              K.QM_B_SIGNED: int(b_dt == "i8"), K.QM_A_ZERO: zero(op.input0_zero_point, "a zero point"),
              K.QM_B_ZERO: zero(op.input1_zero_point, "b zero point"), K.QM_QUANTIZED: int(quantized),
              K.QM_ROWS_PER_BATCH: rpb}
        fp = {}
        if quantized:
            dts = {_suffix(op.input0_scale_dtype), _suffix(op.input1_scale_dtype), _suffix(op.output_scale_dtype)}
            if dts != {"f32"}:
                raise UnsupportedOpError("QLinearMatMul: only fp32 scales")
            sa, sb, sy = (np.float32(self._scalar(nm, "scale")) for nm in
                          (op.input0_scale, op.input1_scale, op.output_scale))
            # the template's float scale ((float)sa * (float)sb / (float)sy) and its integer requant
            # parameters, computed with the same double operations
            scale = np.float32(np.float32(sa * sb) / sy)
            real = float(sa) * float(sb) / float(sy)
            frac = 31
            scaled = math.ldexp(real, frac)
            while frac > 0 and abs(scaled) > 2147483647.0:
                frac -= 1
                scaled = math.ldexp(real, frac)
            mult = int(math.copysign(math.floor(abs(scaled) + 0.5), scaled)) if math.isfinite(scaled) else 0
            if math.isfinite(scaled) and abs(scaled) - math.floor(abs(scaled)) == 0.5:
                mult = int(math.copysign(math.floor(abs(scaled)) + 1, scaled))  # llround: ties away from zero
            rq = math.ldexp(float(mult), -frac)
            use_int = math.isfinite(real) and abs(real - rq) <= max(1e-12, abs(real) * 1e-12)
            ydt = _suffix(op.dtype)
            ip.update({K.QM_USE_INT: int(use_int), K.QM_FRAC_BITS: frac, K.QM_MULT: mult,
                       K.QM_Y_ZERO: int(self._scalar(op.output_zero_point, "y zero point")),
                       K.QM_Y_SIGNED: int(ydt == "i8")})
            fp = {K.QMF_SCALE: float(scale)}
            y = self._dest(op.output, ydt, tuple(op.output_shape))
            kern = K.K_QLINEAR_MATMUL
        else:
            y = self._dest(op.output, "i32", tuple(op.output_shape))
            kern = K.K_MATMUL_INTEGER
        tensors, label = [a, b_, y], f"{op.output} ({what})"
        k, n, m = int(op.k), int(op.n), int(op.m)
        if self.use_tensor_cores and k % 16 == 0 and 16 <= k <= 32768:
            # tcgen05 kind::i8 path: B^T [N][K] (the K-major operand) and B's column sums -- packed
            # once here when B is an initializer, else filled by every run -- and A's row sums
            if op.input1 in self._consts:
                bc = self._consts[op.input1].reshape(k, n)
                tensors += [self._b.weight(np.ascontiguousarray(bc.T).view(np.uint8), "u8",
                                           f"{op.output}:b-transposed"),
                            self._b.weight(bc.astype(np.int64).sum(axis=0).astype(np.int32), "i32",
                                           f"{op.output}:b-column-sums")]
                ip[K.QM_B_PACKED] = 1
            else:
                tensors += [self._b.arena_tensor(T_TEMP, "u8", (n, k), name=f"{op.output}:b-transposed"),
                            self._b.arena_tensor(T_TEMP, "i32", (n,), name=f"{op.output}:b-column-sums")]
            tensors.append(self._b.arena_tensor(T_TEMP, "i32", (m,), name=f"{op.output}:a-row-sums"))
            label += " [tensor cores]"
        self._b.op(kern, tensors, ip, fp, label=label, batched=batched)

    def _emit_QLinearMatMulOp(self, i, op):
        self._emit_matmul8(op, True)

    def _emit_MatMulIntegerOp(self, i, op):
        self._emit_matmul8(op, False)

    # ------------------------------------------------------------------ Conv fp32
    def _emit_ConvOp(self, i, op):
        if _suffix(op.dtype) != "f32" or int(op.spatial_rank) != 2:
            raise UnsupportedOpError("Conv: fp32 2-D only")
        x, w = self._src(op.input0), self._src(op.weights)
        t_b = self._src(op.bias) if op.bias is not None else -1
        n, c = int(op.batch), int(op.in_channels)
        h, wd = op.in_spatial
        oh, ow = op.out_spatial
        y = self._dest(op.output, "f32", (n, int(op.out_channels), oh, ow))
        kh, kw = op.kernel_shape
        # Adding x * w = +-0 for a tap outside the image equals skipping it (the reference
        # skips) unless the accumulator is -0, which needs a -0 bias, or w is inf/NaN
        # (0 * inf = NaN).  With constant weights that rule both out, the kernel may stage
        # zeros for such taps and drop the per-tap test.
        zero_taps_ok = op.weights in self._consts and bool(np.isfinite(self._consts[op.weights]).all())
        if zero_taps_ok and op.bias is not None:
            bias = self._consts.get(op.bias)
            zero_taps_ok = bias is not None and not bool(((bias == 0) & np.signbit(bias)).any())
        self._b.op(K.K_CONV_F32, [x, w, t_b, y], {K.CF_ZERO_TAPS_OK: int(zero_taps_ok),
            K.CF_N: n, K.CF_C: c, K.CF_H: h, K.CF_W: wd, K.CF_OC: int(op.out_channels), K.CF_KH: kh, K.CF_KW: kw,
            K.CF_OH: oh, K.CF_OW: ow, K.CF_SH: op.strides[0], K.CF_SW: op.strides[1], K.CF_PT: op.pads[0],
            K.CF_PL: op.pads[1], K.CF_DH: op.dilations[0], K.CF_DW: op.dilations[1], K.CF_GROUP: int(op.group)},
            label=f"{op.output} (Conv fp32, reference order)",
            batched=self._batch > 0 and n == self._batch and self._is_batched(op.input0))

    # ------------------------------------------------------------------ Softmax fp32
    def _emit_SoftmaxOp(self, i, op):
        if self._dtype(op.input0) != "f32" or getattr(op, "use_legacy_axis_semantics", False):
            raise UnsupportedOpError("Softmax: fp32 with opset-13 axis semantics only")
        shape = tuple(self._shape(op.input0))
        ax = (-1 if op.axis is None else int(op.axis)) % len(shape)
        outer = int(np.prod(shape[:ax]))
        inner = int(np.prod(shape[ax + 1:]))
        x = self._src(op.input0)
        y = self._dest(op.output, "f32", shape)
        batched = self._batch > 0 and ax > 0 and shape[0] == self._batch and self._is_batched(op.input0)
        self._b.op(K.K_SOFTMAX_F32, [x, y], {K.SM_OUTER: outer, K.SM_AXIS: shape[ax], K.SM_INNER: inner,
                                             K.SM_OUTER_PER_BATCH: outer // self._batch if batched else 0},
                   label=f"{op.output} (Softmax fp32)", batched=batched)

    # ------------------------------------------------------------------ layout and pooling
    def _emit_ReshapeOp(self, i, op):
        """The same bytes under another shape: an alias of the source tensor,
        a byte copy only when the result is a graph output."""
        src = self._src(op.input0)
        if op.output not in self._graph_outputs:
            self._nchw[op.output] = src
            return
        shape = tuple(self._shape(op.output))
        nbytes = int(np.prod(shape)) * np.dtype(NP[self._dtype(op.output)]).itemsize
        y = self._dest(op.output, self._dtype(op.output), shape)
        batched = (self._batch > 0 and len(shape) > 0 and shape[0] == self._batch
                   and self._is_batched(op.input0))
        self._b.op(K.K_COPY, [src, y], {K.CP_BYTES: nbytes, K.CP_BATCH: self._batch if batched else 0},
                   label=f"{op.output} (Reshape)", batched=batched)

    def _emit_TransposeOp(self, i, op):
        dt = self._dtype(op.input0)
        elem = np.dtype(NP[dt]).itemsize
        if elem not in (1, 2, 4):
            raise UnsupportedOpError(f"Transpose of {dt} has no B200 kernel")
        shape = tuple(self._shape(op.input0))
        rank = len(shape)
        if rank > 6:
            raise UnsupportedOpError("Transpose: rank above 6 has no B200 kernel")
        perm = tuple(int(p_) for p_ in op.perm)
        strides = [int(np.prod(shape[j + 1:])) for j in range(rank)]
        out_shape = tuple(shape[p_] for p_ in perm)
        pad = 6 - rank
        ip = {K.TR_ELEM: elem, K.TR_BATCH_AXIS: -1}
        for j in range(6):
            ip[K.TR_D0 + j] = out_shape[j - pad] if j >= pad else 1
            ip[K.TR_S0 + j] = strides[perm[j - pad]] if j >= pad else 0
        batched = (self._batch > 0 and rank > 0 and perm[0] == 0 and shape[0] == self._batch
                   and self._is_batched(op.input0))
        if batched:
            ip[K.TR_BATCH_AXIS] = pad
        x = self._src(op.input0)
        y = self._dest(op.output, dt, out_shape)
        self._b.op(K.K_TRANSPOSE, [x, y], ip, label=f"{op.output} (Transpose {perm})", batched=batched)

    def _pool_ip(self, op, kh, kw, sh, sw, dh, dw, pt, pl, oh, ow, xdt, ydt) -> dict:
        n, c, h, w = self._shape(op.input0)
        return {K.PL_N: n, K.PL_C: c, K.PL_H: h, K.PL_W: w, K.PL_OH: oh, K.PL_OW: ow, K.PL_KH: kh, K.PL_KW: kw,
                K.PL_SH: sh, K.PL_SW: sw, K.PL_DH: dh, K.PL_DW: dw, K.PL_PT: pt, K.PL_PL: pl,
                K.PL_X_SIGNED: int(xdt == "i8"), K.PL_Y_SIGNED: int(ydt == "i8")}

    def _emit_MaxPoolOp(self, i, op):
        dt = self._dtype(op.input0)
        if dt not in ("u8", "i8"):
            raise UnsupportedOpError(f"MaxPool on {dt} has no B200 kernel (8-bit only)")
        if op.spatial_rank != 2 or op.indices:
            raise UnsupportedOpError("MaxPool: 2-D pooling without the indices output only")
        ip = self._pool_ip(op, *op.kernel_shape, *op.strides, *op.dilations, op.pads[0], op.pads[1],
                           *op.out_spatial, dt, dt)
        x = self._src(op.input0)
        y = self._dest(op.output, dt, (op.batch, op.channels, *op.out_spatial))
        self._b.op(K.K_MAXPOOL, [x, y], ip, label=f"{op.output} (MaxPool)",
                   batched=op.batch == self._batch and self._is_batched(op.input0))

    def _emit_QLinearAveragePoolOp(self, i, op):
        xdt, ydt = self._dtype(op.input0), self._dtype(op.output)
        if xdt not in ("u8", "i8") or ydt not in ("u8", "i8") or op.channels_last:
            raise UnsupportedOpError("QLinearAveragePool: 8-bit NCHW only")
        if _suffix(op.input_scale_dtype) != "f32" or _suffix(op.output_scale_dtype) != "f32":
            raise UnsupportedOpError("QLinearAveragePool: fp32 scales only")
        xs = np.float32(self._scalar(op.input_scale, "x_scale"))
        ys = np.float32(self._scalar(op.output_scale, "y_scale"))
        ip = self._pool_ip(op, op.kernel_h, op.kernel_w, op.stride_h, op.stride_w, op.dilation_h, op.dilation_w,
                           op.pad_top, op.pad_left, op.out_h, op.out_w, xdt, ydt)
        ip.update({K.PL_COUNT_PAD: int(op.count_include_pad),
                   K.PL_X_ZERO: int(self._scalar(op.input_zero_point, "x_zero_point")),
                   K.PL_Y_ZERO: int(self._scalar(op.output_zero_point, "y_zero_point"))})
        x = self._src(op.input0)
        y = self._dest(op.output, ydt, (op.batch, op.channels, op.out_h, op.out_w))
        self._b.op(K.K_QLINEAR_AVGPOOL, [x, y], ip, {K.PLF_SCALE: float(np.float32(xs / ys))},
                   label=f"{op.output} (QLinearAveragePool)",
                   batched=op.batch == self._batch and self._is_batched(op.input0))

    def _emit_QLinearSoftmaxOp(self, i, op):
        xdt, ydt = self._dtype(op.input0), self._dtype(op.output)
        if xdt not in ("u8", "i8") or ydt != xdt:
            raise UnsupportedOpError("QLinearSoftmax: 8-bit only")
        if _suffix(op.input_scale_dtype) != "f32" or _suffix(op.output_scale_dtype) != "f32":
            raise UnsupportedOpError("QLinearSoftmax: fp32 scales only")
        xs = np.float32(self._scalar(op.input_scale, "x_scale"))
        ys = np.float32(self._scalar(op.output_scale, "y_scale"))
        if not np.isfinite(xs):
            raise UnsupportedOpError("QLinearSoftmax: x_scale must be finite")
        zx = int(self._scalar(op.input_zero_point, "x_zero_point"))
        table = self._b.weight(qsoftmax_exp_table(xdt == "i8", zx, xs), "f32", f"{op.output}:expf-table")
        # ONNX Runtime's floored reciprocal of the output scale, in float
        y_inv = np.floor(np.float32(1.0) / ys).astype(np.float32)
        shape = tuple(op.input_shape)
        batched = (self._batch > 0 and op.axis == 1 and op.outer == self._batch and op.inner == 1
                   and self._is_batched(op.input0))
        x = self._src(op.input0)
        y = self._dest(op.output, ydt, shape)
        self._b.op(K.K_QLINEAR_SOFTMAX, [x, y, table], {
            K.QS_OUTER: op.outer, K.QS_AXIS: op.axis_size, K.QS_INNER: op.inner, K.QS_X_SIGNED: int(xdt == "i8"),
            K.QS_Y_SIGNED: int(ydt == "i8"), K.QS_X_ZERO: zx,
            K.QS_Y_ZERO: int(self._scalar(op.output_zero_point, "y_zero_point"))},
            {K.QSF_X_SCALE: float(xs), K.QSF_Y_INV: float(y_inv)}, label=f"{op.output} (QLinearSoftmax)",
            batched=batched)

    # ------------------------------------------------------------------ Quantize / Dequantize
    def _emit_quant(self, op, quantize: bool):
        what = "QuantizeLinear" if quantize else "DequantizeLinear"
        if getattr(op, "block_size", None):
            raise UnsupportedOpError(f"{what}: blocked quantisation has no B200 kernel")
        shape = tuple(self._shape(op.input0))
        qdt = self._dtype(op.output) if quantize else self._dtype(op.input0)
        if qdt not in ("u8", "i8") or self._dtype(op.scale) != "f32":
            raise UnsupportedOpError(f"{what}: 8-bit data and fp32 scales only")
        if (self._dtype(op.input0) if quantize else self._dtype(op.output)) != "f32":
            raise UnsupportedOpError(f"{what}: fp32 side only")
        sc = self._const(op.scale, "scale").astype(np.float32).reshape(-1)
        if sc.size > 1:
            ax = (1 if op.axis is None else int(op.axis)) % len(shape)
            axis_len, inner = shape[ax], int(np.prod(shape[ax + 1:]))
            if sc.size != axis_len:
                raise UnsupportedOpError(f"{what}: scale length does not match the axis")
        else:
            axis_len, inner = 1, 1
        t_s = self._b.weight(sc, "f32", op.scale)
        t_z = -1
        if op.zero_point is not None:
            z = self._const(op.zero_point, "zero point").reshape(-1)
            t_z = self._b.weight(z.astype(np.int8 if qdt == "i8" else np.uint8), qdt, op.zero_point)
        x = self._src(op.input0)
        y = self._dest(op.output, qdt if quantize else "f32", shape)
        rows = shape[0] if (shape and self._batch > 0 and shape[0] == self._batch and self._is_batched(op.input0)
                            and not (axis_len > 1 and (1 if op.axis is None else int(op.axis)) % len(shape) == 0)) else 0
        self._b.op(K.K_QUANTIZE_LINEAR if quantize else K.K_DEQUANTIZE_LINEAR, [x, t_s, t_z, y],
                   {K.QL_COUNT: int(np.prod(shape)), K.QL_AXIS_LEN: axis_len, K.QL_INNER: inner,
                    K.QL_SIGNED: int(qdt == "i8"), K.QL_ROWS: rows}, label=f"{op.output} ({what})", batched=rows > 0)

    def _emit_QuantizeLinearOp(self, i, op):
        self._emit_quant(op, True)

    def _emit_DequantizeLinearOp(self, i, op):
        self._emit_quant(op, False)

    # ------------------------------------------------------------------ Attention
    def _emit_AttentionOp(self, i, op):
        why = None
        if self._dtype(op.input_q) != "f16" or _suffix(op.dtype) != "f16":
            why = "only fp16"
        elif any(getattr(op, f, None) for f in ("input_attn_mask", "input_past_key", "input_past_value",
                                                 "input_nonpad_kv_seqlen", "output_present_key",
                                                 "output_present_value", "output_qk_matmul")):
            why = "masks, past key/value and extra outputs"
        elif float(op.softcap) != 0.0:
            why = "softcap"
        elif int(op.v_head_size) > 128 or int(op.v_head_size) % 2:
            why = "v head size above 128 or odd"
        if why:
            raise UnsupportedOpError(f"Attention: {why} has no B200 kernel")
        b, hq, hkv = int(op.batch), int(op.q_heads), int(op.kv_heads)
        tq, tk, d, dv = int(op.q_seq), int(op.total_seq), int(op.qk_head_size), int(op.v_head_size)

        def strides(rank, heads, t, hd):
            # 4-D [B][H][T][hd] or 3-D [B][T][H*hd]: (batch, head, token) strides in elements
            return (heads * t * hd, t * hd, hd) if rank == 4 else (t * heads * hd, hd, heads * hd)

        q_rank = int(op.q_rank)
        k_rank = int(getattr(op, "k_rank", q_rank))
        v_rank = int(getattr(op, "v_rank", q_rank))
        o_rank = int(getattr(op, "output_rank", q_rank))
        ss = (*strides(q_rank, hq, tq, d), *strides(k_rank, hkv, int(op.kv_seq), d),
              *strides(v_rank, hkv, int(op.kv_seq), dv), *strides(o_rank, hq, tq, dv))
        q, k, v = self._src(op.input_q), self._src(op.input_k), self._src(op.input_v)
        out_shape = tuple(self._shape(op.output))
        y = self._dest(op.output, "f16", out_shape)
        t_st = self._b.arena_tensor(T_TEMP, "u8", (16,), name="attention:stats")
        # `const _Float16 scale = (_Float16)<float literal>;`: float first, then fp16
        scale16 = float(np.float16(np.float32(float(op.scale))))
        batched = (self._batch > 0 and b == self._batch and self._is_batched(op.input_q)
                   and self._is_batched(op.input_k) and self._is_batched(op.input_v))
        ip = {K.AT_B: b, K.AT_HQ: hq, K.AT_GROUP: hq // hkv, K.AT_TQ: tq, K.AT_TK: tk, K.AT_PAST: int(op.past_seq),
              K.AT_D: d, K.AT_DV: dv, K.AT_CAUSAL: int(bool(op.is_causal))}
        for slot, val in zip(range(K.AT_Q_SB, K.AT_O_ST + 1), ss):
            ip[slot] = val
        tensor = (self.attention_mode == "tensor" and self.use_tensor_cores and d == 128 and dv == 128
                  and all(st % 8 == 0 for st in ss))
        if tensor:
            self._b.op(K.K_ATTENTION_TC, [q, k, v, y, t_st], ip, {K.ATF_SCALE: scale16},
                       label=f"{op.output} (tensor cores, fp32 online softmax)", batched=batched)
        else:
            self._b.op(K.K_ATTENTION_F16, [q, k, v, y, t_st], ip, {K.ATF_SCALE: scale16},
                       label=f"{op.output} (reference fp16 arithmetic)", batched=batched)

    # ------------------------------------------------------------------ LSTM
    def _emit_LstmOp(self, i, op):
        why = None
        if self._dtype(op.input_x) != "f32":
            why = "only fp32"
        elif str(op.direction) != "forward" or int(op.num_directions) != 1:
            why = f"direction {op.direction}"
        elif int(op.layout) != 0:
            why = "layout 1"
        elif op.clip is not None or int(op.input_forget):
            why = "clip / input_forget"
        elif tuple(op.activation_kinds) not in ((), (2, 1, 1)):
            why = "non-default activations"
        elif any(getattr(op, f, None) for f in ("input_sequence_lens", "input_initial_h", "input_initial_c",
                                                 "input_p")):
            why = "sequence_lens / initial_h / initial_c / peepholes"
        elif int(op.input_size) % 4 or int(op.hidden_size) % 4:
            why = "input and hidden sizes must be multiples of 4"
        if why:
            raise UnsupportedOpError(f"LSTM: {why} has no B200 kernel")
        t, b, isz, h = int(op.seq_length), int(op.batch_size), int(op.input_size), int(op.hidden_size)
        w = self._const(op.input_w, "W").astype(np.float32).reshape(4, h, isz)
        r = self._const(op.input_r, "R").astype(np.float32).reshape(4, h, h)
        if op.input_b is not None:
            bb = self._const(op.input_b, "B").astype(np.float32).reshape(8, h)
            bsum = (bb[:4] + bb[4:]).astype(np.float32)  # Wb + Rb, one float add as in the reference
        else:
            bsum = np.zeros((4, h), np.float32)
        # gate columns in tiles of 4 * U: position g*U + u of tile T is gate g (i, o, f, c) of
        # unit T*U + u; units padded to a multiple of U with zero rows
        u = K.LS_TILE_UNITS
        hp = -(-h // u) * u
        order = np.arange(4 * hp)
        tile, pos = order // (4 * u), order % (4 * u)
        gate, unit = pos // u, tile * u + pos % u
        real = unit < h
        wp = np.zeros((4 * hp, isz), np.float32)
        rp = np.zeros((4 * hp, h), np.float32)
        bs = np.zeros(4 * hp, np.float32)
        wp[real] = w[gate[real], unit[real]]
        rp[real] = r[gate[real], unit[real]]
        bs[real] = bsum[gate[real], unit[real]]
        bsum = bs
        t_w = self._b.weight(wp, "f32", op.input_w + ":interleaved")
        t_r = self._b.weight(rp, "f32", op.input_r + ":interleaved")
        t_bs = self._b.weight(bsum, "f32", (op.input_b or "lstm") + ":bias-sum")
        x = self._src(op.input_x)
        # the persistent kernel computes each step's x terms itself; only the
        # per-step path needs every step's x partial sums in the arena
        persistent = lstm_persistent_fits(b, isz, h, K.LP_PLAN_SMS)
        gx_shape = (1, 4) if persistent else (t * b, 4 * hp)
        t_gx = self._b.arena_tensor(T_TEMP, "f32", gx_shape, name=f"{op.input_x}:lstm-x-partials")
        t_h = self._b.arena_tensor(T_TEMP, "f32", (2, b, h), name="lstm:h")
        t_c = self._b.arena_tensor(T_TEMP, "f32", (b, h), name="lstm:c")
        outs = []
        for name, shp in ((op.output_y, (t, 1, b, h)), (op.output_y_h, (1, b, h)), (op.output_y_c, (1, b, h))):
            outs.append(self._dest(name, "f32", shp) if name else -1)
        self._b.op(K.K_LSTM_F32, [x, t_w, t_r, t_bs, t_gx, t_h, t_c, *outs],
                   {K.LS_T: t, K.LS_B: b, K.LS_I: isz, K.LS_H: h, K.LS_GX_PLACEHOLDER: int(persistent)},
                   label=f"LSTM T={t} B={b} I={isz} H={h} (reference order, "
                         f"{'one persistent launch' if persistent else 'one launch per step'})")

    # ------------------------------------------------------------------ MatMulNBits
    def _nbits_reject(self, op) -> str | None:
        """Why this MatMulNBits has no tensor-core kernel (None: it has one)."""
        if int(op.bits) != 4:
            return f"{op.bits}-bit weights"
        if self._dtype(op.input0) != "f16" or _suffix(op.output_dtype) != "f16":
            return "only fp16 activations and outputs"
        if int(op.accuracy_level) == 4:
            return "accuracy_level 4 (int8 activation path)"
        bs = int(op.block_size)
        if bs < 16 or bs & (bs - 1):
            return f"block_size {bs}"
        if int(op.k) % 8 or int(op.n) % 8:
            return "K and N must be multiples of 8 (16-byte row pitches)"
        for what, name in (("B", op.input1), ("scales", op.scales), ("zero_points", op.zero_points),
                           ("bias", op.bias)):
            if name is not None and name not in self._consts:
                return f"{what} must be an initializer"
        if self._dtype(op.scales) != "f16":
            return "only fp16 scales"
        if op.zero_points is not None and self._dtype(op.zero_points) != "u8":
            return "only packed uint8 zero points"
        return None

    def _nbits_part(self, op):
        n, k, bs = int(op.n), int(op.k), int(op.block_size)
        n_blocks = -(-k // bs)
        q = unpack_nbits(self._consts[op.input1], n, bs)
        zp = unpack_nbits_zero_points(self._consts[op.zero_points] if op.zero_points else None, n, n_blocks)
        sc = np.asarray(self._consts[op.scales], np.float16).reshape(n, -1)
        if sc.shape[1] == 1 and n_blocks > 1:
            sc = np.repeat(sc, n_blocks, axis=1)
        bias = np.asarray(self._consts[op.bias], np.float16).astype(np.float32).reshape(-1) if op.bias else None
        return q, zp, sc, bias

    def _nbits_emit(self, ops_, out_name, fused_alpha=None):
        g = ops_[0]
        k, n = int(g.k), int(g.n)
        a_shape = tuple(self._shape(g.input0))
        rows = int(np.prod(a_shape[:-1])) if len(a_shape) > 1 else 1
        img, bias, n_tiles, k_steps, groups = nbits_weight_image(
            [self._nbits_part(o) for o in ops_], k, int(g.block_size), fused_alpha is not None)
        t_w = self._b.weight(img, "u8", g.input1 + ":tc")
        t_b = self._b.weight(bias, "f32", g.output + ":bias") if bias is not None else -1
        a = self._src(g.input0)
        out_shape = a_shape[:-1] + (n,)
        y = self._dest(out_name, "f16", out_shape)
        batched = (len(a_shape) > 1 and a_shape[0] == self._batch and self._batch > 0
                   and self._is_batched(g.input0))
        ip = {K.NB_ROWS: rows, K.NB_K: k, K.NB_N_OUT: n, K.NB_KSTEPS: k_steps, K.NB_NTILES: n_tiles,
              K.NB_GROUPS: groups, K.NB_FUSED: int(fused_alpha is not None), K.NB_A_PITCH: k, K.NB_Y_PITCH: n,
              K.NB_ROWS_PER_BATCH: rows // self._batch if batched else 0,
              K.NB_ROUNDED_DEQUANT: int(self.nbits_rounded_dequant)}
        fp = {K.NBF_ALPHA: float(fused_alpha if fused_alpha is not None else 1.0)}
        label = (f"{ops_[0].output}, {ops_[1].output} -> Swish * Mul -> {out_name} (tcgen05 f16, fused)"
                 if fused_alpha is not None else f"{out_name} (tcgen05 f16)")
        self._b.op(K.K_NBITS_GEMM, [a, t_w, t_b, y], ip, fp, label=label, batched=batched)

    def _nbits_i8_reject(self, op) -> str | None:
        """Why an accuracy_level-4 MatMulNBits has no int8-path kernel (None: it has one)."""
        if int(op.bits) != 4:
            return f"{op.bits}-bit weights on the int8 activation path"
        if self._dtype(op.input0) != "f16" or _suffix(op.output_dtype) != "f16":
            return "only fp16 activations and outputs on the int8 activation path"
        bs = int(op.block_size)
        if bs < 16 or bs % 16 or bs > 4096:
            return f"block_size {bs} on the int8 activation path"
        for what, name in (("B", op.input1), ("scales", op.scales), ("zero_points", op.zero_points),
                           ("bias", op.bias)):
            if name is not None and name not in self._consts:
                return f"{what} must be an initializer"
        if op.zero_points is not None and self._dtype(op.zero_points) != "u8":
            return "only packed uint8 zero points on the int8 activation path"
        if op.bias is not None and self._dtype(op.bias) != "f16":
            return "only fp16 bias"
        return None

    def _nbits_i8_emit(self, op):
        """accuracy_level 4 (templates/matmul_nbits_int8_op.c.j2): weights packed
        as int8 (q - zp) [N][KP] with KP the K blocks' padded length (zeros past
        K, so a partial last block adds exact zeros), scales as float
        [N][n_blocks]; the quantised activations and their block scales are
        per-run scratch."""
        n, k, bs = int(op.n), int(op.k), int(op.block_size)
        nblk = -(-k // bs)
        kp = nblk * bs
        q, zp, sc, bias = self._nbits_part(op)
        w = np.zeros((n, kp), np.int8)
        w[:, :k] = (q[:, :k].astype(np.int16) - np.repeat(zp.astype(np.int16), bs, axis=1)[:, :k]).astype(np.int8)
        t_w = self._b.weight(w, "i8", op.input1 + ":int8-minus-zp")
        t_s = self._b.weight(np.ascontiguousarray(sc.astype(np.float32)), "f32", op.scales + ":f32")
        t_b = self._b.weight(bias, "f32", op.bias + ":f32") if bias is not None else -1
        a = self._src(op.input0)
        a_shape = tuple(self._shape(op.input0))
        rows = int(np.prod(a_shape[:-1])) if len(a_shape) > 1 else 1
        t_qa = self._b.arena_tensor(T_TEMP, "i8", (rows, kp), name=f"{op.output}:int8-activations")
        t_as = self._b.arena_tensor(T_TEMP, "f32", (rows, nblk), name=f"{op.output}:activation-block-scales")
        y = self._dest(op.output, "f16", a_shape[:-1] + (n,))
        batched = (len(a_shape) > 1 and a_shape[0] == self._batch and self._batch > 0
                   and self._is_batched(op.input0))
        ip = {K.NI_ROWS: rows, K.NI_K: k, K.NI_KP: kp, K.NI_N: n, K.NI_BLOCK: bs, K.NI_NBLK: nblk,
              K.NI_ROWS_PER_BATCH: rows // self._batch if batched else 0}
        self._b.op(K.K_NBITS_I8, [a, t_w, t_s, t_b, t_qa, t_as, y], ip,
                   label=f"{op.output} (int8 activations, accuracy_level 4)", batched=batched)

    def _emit_MatMulNBitsOp(self, i, op):
        if i in self._nbits_fused:
            f = self._nbits_fused[i]
            return self._nbits_emit([f["gate"], f["up"]], f["mul"].output, fused_alpha=f["alpha"])
        if int(op.accuracy_level) == 4:
            why = self._nbits_i8_reject(op)
            if why:
                raise UnsupportedOpError(f"MatMulNBits: {why}")
            return self._nbits_i8_emit(op)
        why = self._nbits_reject(op)
        if why:
            raise UnsupportedOpError(f"MatMulNBits: {why}")
        self._nbits_emit([op], op.output)


# ------------------------------------------------------------------ plan files
def save_plan(plan: Plan, out_dir, stem: str | None = None) -> dict:
    """Write ``<stem>.plan`` (the launch plan), ``<stem>.weights`` (the packed
    weight blob, read by emx_b200_plan_load) and ``<stem>.json`` (graph I/O
    names, shapes and dtypes, batch, op labels).  Returns the paths."""
    import json
    from pathlib import Path
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    stem = stem or plan.name
    paths = {k: out / f"{stem}.{k}" for k in ("plan", "weights", "json")}
    paths["plan"].write_bytes(plan.plan_bytes)
    paths["weights"].write_bytes(plan.weight_bytes)
    meta = {
        "name": plan.name, "batch": plan.batch, "arena_bytes": plan.arena_bytes,
        "inputs": [{"name": n, "shape": list(s), "dtype": d}
                   for n, s, d in zip(plan.input_names, plan.input_shapes, plan.input_dtypes)],
        "outputs": [{"name": n, "shape": list(s), "dtype": d}
                    for n, s, d in zip(plan.output_names, plan.output_shapes, plan.output_dtypes)],
        "ops": [f"{K.NAMES.get(op.kernel, op.kernel)}: {op.label}" for op in plan.ops],
    }
    paths["json"].write_text(json.dumps(meta, indent=1) + "\n")
    return paths


def load_plan(prefix) -> tuple[Plan, str]:
    """Read the files written by save_plan (``prefix`` without extension):
    the Plan (without its weight blob) and the weights file path for
    Session(plan, weights_path=...)."""
    import json
    from pathlib import Path
    prefix = Path(prefix)
    meta = json.loads(prefix.with_suffix(".json").read_text())
    plan_bytes = prefix.with_suffix(".plan").read_bytes()
    ins, outs = meta["inputs"], meta["outputs"]
    plan = Plan(meta["name"], plan_bytes, b"", tuple(t["name"] for t in ins), tuple(tuple(t["shape"]) for t in ins),
                tuple(t["dtype"] for t in ins), tuple(t["name"] for t in outs),
                tuple(tuple(t["shape"]) for t in outs), tuple(t["dtype"] for t in outs), int(meta["batch"]),
                [PlanOp(0, [], label=s) for s in meta["ops"]], [], int(meta["arena_bytes"]))
    return plan, str(prefix.with_suffix(".weights"))
