"""Network definitions in ONNX/ENNF terms, with seeded synthetic weights.

A :class:`Graph` is an ordered ONNX-style graph (named tensors, initializers, nodes with
attributes, full static shapes for every intermediate).  It is the single source for the
two serialisations this project needs:

* ``spinn_b200.ennf.convert`` -- the fused ``.ennf`` file that SPINN's converter
  (``SPINN/onnx2ennf.c`` + ``SPINN/graph_opt.c``) would write for the same graph;
* ``oracle/onnx_writer.py`` -- an ONNX protobuf, fed to the reference converter itself
  (test infrastructure) to pin the former byte for byte.

Node order follows a PyTorch ``torch.onnx`` export (conv, bn, relu, ...), because the
reference fusion passes are order sensitive (``SPINN/graph_opt.c:350-374``).

Synthetic data follows the benchmark configurations: conv weights He-normal
``N(0, sqrt(2/fan_in))``, BatchNorm ``gamma~U(0.5,1.5)``, ``beta,mean~N(0,0.1)``,
``var~U(0.5,1.5)``, ``eps=1e-5``; all parameters drawn from one
``numpy.random.default_rng(seed)`` in node order (conv weight, then gamma, beta, mean,
var); the FC layer ``W,b ~ U(-1/sqrt(fan_in), 1/sqrt(fan_in))``.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

Shape = Tuple[int, ...]


@dataclass
class Node:
    op_type: str
    inputs: List[str]
    outputs: List[str]
    attrs: Dict[str, object] = field(default_factory=dict)
    name: str = ""


@dataclass
class Graph:
    name: str = "spinn_b200"
    nodes: List[Node] = field(default_factory=list)
    initializers: Dict[str, np.ndarray] = field(default_factory=dict)
    inputs: List[Tuple[str, Shape]] = field(default_factory=list)
    outputs: List[Tuple[str, Shape]] = field(default_factory=list)
    value_info: Dict[str, Shape] = field(default_factory=dict)
    opset: int = 13
    # ONNX element type of non-initializer tensors that are not float32 (7 = int64)
    elem_types: Dict[str, int] = field(default_factory=dict)

    # ------------------------------------------------------------------ helpers
    def shape(self, name: str) -> Shape:
        if name in self.initializers:
            return tuple(self.initializers[name].shape)
        for n, s in self.inputs:
            if n == name:
                return s
        return self.value_info[name]

    def add_input(self, name: str, shape: Sequence[int]) -> str:
        self.inputs.append((name, tuple(int(d) for d in shape)))
        return name

    def add_init(self, name: str, arr: np.ndarray) -> str:
        arr = np.asarray(arr)
        dt = np.int64 if arr.dtype.kind in "iu" else np.float32
        self.initializers[name] = np.ascontiguousarray(arr, dtype=dt)
        return name

    def add_node(self, op: str, inputs: Sequence[str], outputs: Sequence[str],
                 out_shapes: Sequence[Shape], out_types: Optional[Sequence[int]] = None, **attrs) -> List[str]:
        for i, (o, s) in enumerate(zip(outputs, out_shapes)):
            self.value_info[o] = tuple(int(d) for d in s)
            if out_types is not None and out_types[i] != 1:
                self.elem_types[o] = int(out_types[i])
        self.nodes.append(Node(op, list(inputs), list(outputs), dict(attrs),
                               name=f"{op}_{len(self.nodes)}"))
        return list(outputs)

    def mark_output(self, name: str) -> None:
        self.outputs.append((name, self.value_info[name]))
        # graph outputs are described by graph.output, not value_info (ONNX convention)
        del self.value_info[name]

    def copy(self) -> "Graph":
        g = Graph(self.name, [Node(n.op_type, list(n.inputs), list(n.outputs), dict(n.attrs), n.name)
                              for n in self.nodes],
                  {k: v.copy() for k, v in self.initializers.items()},
                  list(self.inputs), list(self.outputs), dict(self.value_info), self.opset,
                  dict(self.elem_types))
        return g

    def flops(self) -> int:
        """Algorithmic multiply-add FLOPs (2 per MAC) of the Conv/Gemm/MatMul nodes."""
        total = 0
        for n in self.nodes:
            if n.op_type == "Conv":
                w = self.shape(n.inputs[1])
                y = self._out_shape(n)
                total += 2 * int(np.prod(y)) * w[1] * w[2] * w[3]
            elif n.op_type == "Gemm":
                a = self.shape(n.inputs[0])
                y = self._out_shape(n)
                k = a[0] if n.attrs.get("transA", 0) else a[1]
                total += 2 * y[0] * y[1] * k
            elif n.op_type == "MatMul":
                a = self.shape(n.inputs[0])
                y = self._out_shape(n)
                total += 2 * int(np.prod(y)) * a[-1]
        return total

    def _out_shape(self, n: Node) -> Shape:
        o = n.outputs[0]
        for name, s in self.outputs:
            if name == o:
                return s
        return self.value_info[o]


def conv_out_hw(h: int, w: int, k: int, s: int, p: int) -> Tuple[int, int]:
    return (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1


class _Builder:
    """Small helper that names tensors and draws weights in node order."""

    def __init__(self, g: Graph, rng: np.random.Generator, bn_spread: Optional[float] = None):
        self.g = g
        self.rng = rng
        self.k = 0
        self.bn_spread = bn_spread

    def _id(self, prefix: str) -> str:
        self.k += 1
        return f"{prefix}_{self.k}"

    def conv(self, x: str, oc: int, k: int, s: int, p: int, group: int = 1,
             bias: bool = False, dilation: int = 1) -> str:
        n, c, h, w = self.g.shape(x)
        fan_in = (c // group) * k * k
        wname = self.g.add_init(self._id("conv_w"),
                                self.rng.normal(0.0, np.sqrt(2.0 / fan_in), (oc, c // group, k, k)))
        ins = [x, wname]
        if bias:
            ins.append(self.g.add_init(self._id("conv_b"), self.rng.normal(0.0, 0.1, (oc,))))
        oh, ow = conv_out_hw(h, w, (k - 1) * dilation + 1, s, p)
        return self.g.add_node("Conv", ins, [self._id("conv")], [(n, oc, oh, ow)],
                               kernel_shape=[k, k], strides=[s, s], pads=[p, p, p, p],
                               dilations=[dilation, dilation], group=group)[0]

    def bn(self, x: str, eps: float = 1e-5) -> str:
        c = self.g.shape(x)[1]
        if self.bn_spread is None:   # the benchmark configurations' distribution
            gamma = self.rng.uniform(0.5, 1.5, (c,))
            beta = self.rng.normal(0.0, 0.1, (c,))
            mean = self.rng.normal(0.0, 0.1, (c,))
            var = self.rng.uniform(0.5, 1.5, (c,))
        else:                        # statistics close to an identity normalisation
            e = self.bn_spread
            gamma = self.rng.uniform(1 - e, 1 + e, (c,))
            beta = self.rng.normal(0.0, e, (c,))
            mean = self.rng.normal(0.0, e, (c,))
            var = self.rng.uniform(1 - e, 1 + e, (c,))
        gamma = self.g.add_init(self._id("bn_gamma"), gamma)
        beta = self.g.add_init(self._id("bn_beta"), beta)
        mean = self.g.add_init(self._id("bn_mean"), mean)
        var = self.g.add_init(self._id("bn_var"), var)
        return self.g.add_node("BatchNormalization", [x, gamma, beta, mean, var], [self._id("bn")],
                               [self.g.shape(x)], epsilon=float(eps), momentum=0.9)[0]

    def unary(self, op: str, x: str) -> str:
        return self.g.add_node(op, [x], [self._id(op.lower())], [self.g.shape(x)])[0]

    def add(self, a: str, b: str) -> str:
        return self.g.add_node("Add", [a, b], [self._id("add")], [self.g.shape(a)])[0]

    def mul(self, a: str, b: str) -> str:
        return self.g.add_node("Mul", [a, b], [self._id("mul")], [self.g.shape(a)])[0]

    def silu(self, x: str) -> str:
        s = self.unary("Sigmoid", x)
        return self.mul(x, s)

    def maxpool(self, x: str, k: int, s: int, p: int) -> str:
        n, c, h, w = self.g.shape(x)
        oh, ow = conv_out_hw(h, w, k, s, p)
        return self.g.add_node("MaxPool", [x], [self._id("maxpool")], [(n, c, oh, ow)],
                               kernel_shape=[k, k], strides=[s, s], pads=[p, p, p, p])[0]

    def gap(self, x: str) -> str:
        n, c, _, _ = self.g.shape(x)
        return self.g.add_node("GlobalAveragePool", [x], [self._id("gap")], [(n, c, 1, 1)])[0]

    def flatten(self, x: str) -> str:
        s = self.g.shape(x)
        return self.g.add_node("Flatten", [x], [self._id("flatten")],
                               [(s[0], int(np.prod(s[1:])))], axis=1)[0]

    def conv_bn(self, x: str, oc: int, k: int, s: int, act: str = "SiLU", group: int = 1) -> str:
        """Conv (no bias) + BatchNorm + activation ("SiLU", "Relu" or None)."""
        y = self.bn(self.conv(x, oc, k, s, k // 2, group=group))
        if act == "SiLU":
            y = self.silu(y)
        elif act == "Relu":
            y = self.unary("Relu", y)
        return y

    def split2(self, x: str):
        n, c, h, w = self.g.shape(x)
        return self.g.add_node("Split", [x], [self._id("split"), self._id("split")],
                               [(n, c // 2, h, w)] * 2, axis=1)

    def concat(self, xs, axis: int = 1) -> str:
        shp = list(self.g.shape(xs[0]))
        shp[axis] = sum(self.g.shape(x)[axis] for x in xs)
        return self.g.add_node("Concat", list(xs), [self._id("concat")], [tuple(shp)], axis=axis)[0]

    def upsample2(self, x: str) -> str:
        n, c, h, w = self.g.shape(x)
        sc = self.g.add_init(self._id("scales"), np.array([1, 1, 2, 2], np.float32))
        return self.g.add_node("Resize", [x, sc], [self._id("resize")], [(n, c, 2 * h, 2 * w)],
                               mode="nearest")[0]

    def reshape(self, x: str, shape) -> str:
        shp = self.g.add_init(self._id("shape"), np.array(shape, np.int64))
        return self.g.add_node("Reshape", [x, shp], [self._id("reshape")], [tuple(shape)])[0]

    def transpose(self, x: str, perm) -> str:
        s = self.g.shape(x)
        return self.g.add_node("Transpose", [x], [self._id("transpose")], [tuple(s[p] for p in perm)],
                               perm=list(perm))[0]

    def matmul(self, a: str, b: str) -> str:
        sa, sb = self.g.shape(a), self.g.shape(b)
        return self.g.add_node("MatMul", [a, b], [self._id("matmul")], [tuple(sa[:-1]) + (sb[-1],)])[0]

    def softmax(self, x: str) -> str:
        return self.g.add_node("Softmax", [x], [self._id("softmax")], [self.g.shape(x)], axis=-1)[0]

    def topk(self, x: str, k: int, axis: int = -1):
        """ONNX TopK (largest, sorted) over the last axis: returns (values, int64 indices)."""
        s = self.g.shape(x)
        kk = self.g.add_init(self._id("k"), np.array([k], np.int64))
        out = tuple(s[:-1]) + (min(k, s[-1]),)
        v, i = self.g.add_node("TopK", [x, kk], [self._id("topk_v"), self._id("topk_i")], [out, out],
                               out_types=[1, 7], axis=axis, largest=1, sorted=1)
        return v, i

    def scale(self, x: str, v: float) -> str:
        c = self.g.add_init(self._id("scale"), np.array([v], np.float32))
        return self.g.add_node("Mul", [x, c], [self._id("mul")], [self.g.shape(x)])[0]

    def gemm(self, x: str, n_out: int, trans_b: int = 1) -> str:
        m, k = self.g.shape(x)
        bound = 1.0 / np.sqrt(k)
        wshape = (n_out, k) if trans_b else (k, n_out)
        w = self.g.add_init(self._id("fc_w"), self.rng.uniform(-bound, bound, wshape))
        b = self.g.add_init(self._id("fc_b"), self.rng.uniform(-bound, bound, (n_out,)))
        return self.g.add_node("Gemm", [x, w, b], [self._id("gemm")], [(m, n_out)],
                               alpha=1.0, beta=1.0, transA=0, transB=int(trans_b))[0]


# ---------------------------------------------------------------------- models
def conv_bn_relu(batch: int = 1, c: int = 64, hw: int = 56, oc: int = 64, k: int = 3,
                 stride: int = 1, pad: int = 1, seed: int = 0, act: str = "Relu", group: int = 1
                 ) -> Tuple[Graph, np.ndarray]:
    """Single Conv+BatchNorm(+act) layer (the benchmark's first configuration; ``group`` > 1
    gives grouped / depthwise layers).

    Draw order from ``default_rng(seed)``: input X~U(-1,1), W~N(0,sqrt(2/fan_in)),
    gamma, beta, mean, var.  Returns the graph and the input tensor.
    """
    rng = np.random.default_rng(seed)
    x_val = rng.uniform(-1.0, 1.0, (batch, c, hw, hw)).astype(np.float32)
    g = Graph("conv_bn_relu")
    b = _Builder(g, rng)
    x = g.add_input("input", (batch, c, hw, hw))
    y = b.bn(b.conv(x, oc, k, stride, pad, group=group))
    if act == "Relu":
        y = b.unary("Relu", y)
    elif act == "SiLU":
        y = b.silu(y)
    g.mark_output(y)
    return g, x_val


def conv_bn_add_relu(batch: int = 1, c: int = 64, hw: int = 56, seed: int = 0
                     ) -> Tuple[Graph, np.ndarray]:
    """Conv+BN whose output is added to the block input and ReLU'd (residual fusion)."""
    rng = np.random.default_rng(seed)
    x_val = rng.uniform(-1.0, 1.0, (batch, c, hw, hw)).astype(np.float32)
    g = Graph("conv_bn_add_relu")
    b = _Builder(g, rng)
    x = g.add_input("input", (batch, c, hw, hw))
    r = b.unary("Relu", x)
    y = b.unary("Relu", b.add(b.bn(b.conv(r, c, 3, 1, 1)), r))
    g.mark_output(y)
    return g, x_val


def conv_bn_proj_add_relu(batch: int = 1, c: int = 256, hw: int = 14, oc: int = 1024, k: int = 1,
                          seed: int = 0) -> Tuple[Graph, np.ndarray]:
    """The last convolution of a bottleneck with a projection shortcut: the shortcut
    BN(Conv1x1(x)) is added to BN(Conv kxk(x)) and ReLU'd, so the second convolution carries
    the fused residual (c -> oc channels, stride 1)."""
    rng = np.random.default_rng(seed)
    x_val = rng.uniform(-1.0, 1.0, (batch, c, hw, hw)).astype(np.float32)
    g = Graph("conv_bn_proj_add_relu")
    b = _Builder(g, rng)
    x = g.add_input("input", (batch, c, hw, hw))
    r = b.bn(b.conv(x, oc, 1, 1, 0))
    y = b.unary("Relu", b.add(b.bn(b.conv(x, oc, k, 1, k // 2)), r))
    g.mark_output(y)
    return g, x_val


RESNET_DEPTHS = {18: None, 50: [3, 4, 6, 3], 101: [3, 4, 23, 3], 152: [3, 8, 36, 3]}


def bottleneck_tail(batch: int, hw: int, n1: int, k1: int, n2: int, relu_reduce: bool = True,
                    seed: int = 11) -> Tuple[Graph, np.ndarray]:
    """The end of one bottleneck block and the start of the next, on their own:
    x [n1 channels] -> 1x1 (n1 -> k1)+BN+ReLU -> 1x1 (k1 -> n1)+BN, + x, ReLU -> 1x1 (n1 -> n2)
    +BN (+ReLU) -> output.  The last two convolutions are the pair the bottleneck-tail kernel
    fuses.  Input N(0, 1) from the same generator, after the weights."""
    rng = np.random.default_rng(seed)
    g = Graph("bottleneck_tail")
    b = _Builder(g, rng)
    x = g.add_input("input", (batch, n1, hw, hw))
    t2 = b.unary("Relu", b.bn(b.conv(x, k1, 1, 1, 0)))
    y = b.unary("Relu", b.add(b.bn(b.conv(t2, n1, 1, 1, 0)), x))
    t = b.bn(b.conv(y, n2, 1, 1, 0))
    if relu_reduce:
        t = b.unary("Relu", t)
    g.mark_output(t)
    return g, rng.standard_normal((batch, n1, hw, hw)).astype(np.float32)


def resnet(depth: int = 50, batch: int = 1, image: int = 224, num_classes: int = 1000,
           seed: int = 2, width: int = 64) -> Graph:
    """Bottleneck ResNet (v1.5: stride on the 3x3 conv), torchvision export order."""
    blocks = RESNET_DEPTHS[depth]
    if blocks is None:
        raise ValueError("only bottleneck depths (50/101/152) are defined")
    rng = np.random.default_rng(seed)
    g = Graph(f"resnet{depth}")
    b = _Builder(g, rng)
    x = g.add_input("input", (batch, 3, image, image))
    y = b.unary("Relu", b.bn(b.conv(x, width, 7, 2, 3)))
    y = b.maxpool(y, 3, 2, 1)
    in_c = width
    for stage, nblk in enumerate(blocks):
        mid = width * (2 ** stage)
        out_c = mid * 4
        for i in range(nblk):
            stride = 2 if (i == 0 and stage > 0) else 1
            idn = y
            t = b.unary("Relu", b.bn(b.conv(y, mid, 1, 1, 0)))
            t = b.unary("Relu", b.bn(b.conv(t, mid, 3, stride, 1)))
            t = b.bn(b.conv(t, out_c, 1, 1, 0))
            if i == 0:
                idn = b.bn(b.conv(y, out_c, 1, stride, 0))
            y = b.unary("Relu", b.add(t, idn))
            in_c = out_c
    y = b.flatten(b.gap(y))
    y = b.gemm(y, num_classes, trans_b=1)
    g.mark_output(y)
    return g


def image_batch(start: int, count: int, image: int = 224, seed: int = 3) -> np.ndarray:
    """Images ``start .. start+count-1`` of a global N(0,1) batch, image i drawn from
    ``default_rng([seed, i])``: a rank's shard equals the slice of the global batch."""
    out = np.empty((count, 3, image, image), np.float32)
    for j in range(count):
        out[j] = np.random.default_rng([seed, start + j]).standard_normal((3, image, image), dtype=np.float32)
    return out


def resnet_input(batch: int, image: int = 224, seed: int = 2) -> np.ndarray:
    """N(0,1) NCHW input, drawn from ``default_rng(seed + 1)``."""
    return np.random.default_rng(seed + 1).standard_normal((batch, 3, image, image),
                                                           dtype=np.float32)


def gemm_case(m: int, n: int, k: int, trans_a: int = 0, trans_b: int = 0, alpha: float = 1.0,
              beta: float = 1.0, c_shape: Optional[str] = "vector", seed: int = 1
              ) -> Tuple[Graph, np.ndarray]:
    """Standalone Gemm ``Y = alpha*A*B + beta*C`` with A, B, C ~ U(-1,1) from ``default_rng(seed)``.

    ``c_shape`` is ``"vector"`` ([N]), ``"full"`` ([M,N]) or ``None`` (no C input).
    B and C are initializers (weights); A is the graph input.
    """
    rng = np.random.default_rng(seed)
    a_val = rng.uniform(-1, 1, (k, m) if trans_a else (m, k)).astype(np.float32)
    g = Graph("gemm")
    a = g.add_input("A", a_val.shape)
    bw = g.add_init("B", rng.uniform(-1, 1, (n, k) if trans_b else (k, n)))
    ins = [a, bw]
    if c_shape == "vector":
        ins.append(g.add_init("C", rng.uniform(-1, 1, (n,))))
    elif c_shape == "full":
        ins.append(g.add_init("C", rng.uniform(-1, 1, (m, n))))
    g.add_node("Gemm", ins, ["Y"], [(m, n)], alpha=float(alpha), beta=float(beta),
               transA=int(trans_a), transB=int(trans_b))
    g.mark_output("Y")
    return g, a_val


# ------------------------------------------------------------------ YOLOv10n-shaped detector
def _c2f(b: _Builder, x: str, c_out: int, n: int, shortcut: bool) -> str:
    """CSP block: 1x1 conv to 2h channels, split in halves, n bottlenecks (two 3x3 convs,
    optional identity shortcut) on the second half, concat of every stage, 1x1 conv."""
    h = c_out // 2
    a, y = b.split2(b.conv_bn(x, 2 * h, 1, 1))
    outs = [a, y]
    for _ in range(n):
        t = b.conv_bn(b.conv_bn(y, h, 3, 1), h, 3, 1)
        y = b.add(y, t) if shortcut else t
        outs.append(y)
    return b.conv_bn(b.concat(outs), c_out, 1, 1)


def _down(b: _Builder, x: str, c_out: int) -> str:
    """Pointwise conv then depthwise 3x3 stride 2 (BN, no activation)."""
    y = b.conv_bn(x, c_out, 1, 1)
    return b.conv_bn(y, c_out, 3, 2, act=None, group=c_out)


def _sppf(b: _Builder, x: str) -> str:
    c = b.g.shape(x)[1]
    y = b.conv_bn(x, c // 2, 1, 1)
    m1 = b.maxpool(y, 5, 1, 2)
    m2 = b.maxpool(m1, 5, 1, 2)
    m3 = b.maxpool(m2, 5, 1, 2)
    return b.conv_bn(b.concat([y, m1, m2, m3]), c, 1, 1)


def _psa(b: _Builder, x: str, heads: int = 2) -> str:
    """Split-attention block: half of the channels pass through self-attention over the
    spatial positions (q, k, v from one 1x1 conv; softmax(q^T k / sqrt(d)) applied to v;
    1x1 projection, residual) and a two-layer 1x1 feed-forward (residual)."""
    n, c, hh, ww = b.g.shape(x)
    a, y = b.split2(b.conv_bn(x, c, 1, 1))
    d = c // 2
    hd = d // heads
    qkv = b.conv_bn(y, 3 * d, 1, 1, act=None)
    q, k, v = (b.reshape(t, (n, heads, hd, hh * ww)) for t in _split3(b, qkv))
    attn = b.softmax(b.scale(b.matmul(b.transpose(q, (0, 1, 3, 2)), k), float(hd) ** -0.5))
    o = b.matmul(v, b.transpose(attn, (0, 1, 3, 2)))
    o = b.reshape(o, (n, d, hh, ww))
    y = b.add(b.conv_bn(o, d, 1, 1, act=None), y)
    y = b.add(b.conv_bn(b.conv_bn(y, 2 * d, 1, 1), d, 1, 1, act=None), y)
    return b.conv_bn(b.concat([a, y]), c, 1, 1)


def _split3(b: _Builder, x: str):
    n, c, h, w = b.g.shape(x)
    return b.g.add_node("Split", [x], [b._id("split") for _ in range(3)], [(n, c // 3, h, w)] * 3, axis=1)


def _head(b: _Builder, x: str, reg: int = 64, nc: int = 80) -> str:
    """Decoupled head: box branch (two 3x3 convs, 1x1 to reg) and class branch (depthwise
    3x3 + pointwise twice, 1x1 to nc), concatenated and flattened to [N, reg+nc, H*W]."""
    n, c, h, w = b.g.shape(x)
    cb = max(16, c // 4, reg // 4)
    bx = b.conv(b.conv_bn(b.conv_bn(x, cb, 3, 1), cb, 3, 1), reg, 1, 1, 0, bias=True)
    cc = max(c, min(nc, 100))
    cl = b.conv_bn(b.conv_bn(x, c, 3, 1, group=c), cc, 1, 1)
    cl = b.conv_bn(b.conv_bn(cl, cc, 3, 1, group=cc), cc, 1, 1)
    cl = b.conv(cl, nc, 1, 1, 0, bias=True)
    return b.reshape(b.concat([bx, cl]), (n, reg + nc, h * w))


YOLO_STAGES = ("stem", "p3", "p4", "c5", "sppf", "psa", "top", "s3", "s4", "s5", "heads")


def yolo_shaped(batch: int = 1, image: int = 640, seed: int = 4, widths=(16, 32, 64, 128, 256),
                depths=(1, 2, 2, 1), nc: int = 80, upto: Optional[str] = None,
                bn_spread: Optional[float] = 0.1) -> Graph:
    """A YOLOv10n-shaped detector: CSP/C2f backbone with pointwise + depthwise-3x3 stride-2
    downsampling and SiLU activations, SPPF pooling, a split-attention (PSA) block, a
    top-down/bottom-up feature pyramid with nearest upsampling and concatenation, and
    decoupled heads at strides 8, 16 and 32, concatenated to [N, 64 + nc, anchors].
    This is a synthetic network of that family (the original configuration is not part of
    the reference); widths/depths follow the family's smallest ("n") scale.  ``upto`` ends
    the graph after one of ``YOLO_STAGES`` (layer-wise parity checks)."""
    if upto is not None and upto not in YOLO_STAGES:
        raise ValueError(upto)
    rng = np.random.default_rng(seed)
    g = Graph(f"yolo_shaped_{image}")
    b = _Builder(g, rng, bn_spread)
    w0, w1, w2, w3, w4 = widths
    x = g.add_input("images", (batch, 3, image, image))

    def done(t: str) -> Graph:
        g.mark_output(t)
        return g

    y = b.conv_bn(x, w0, 3, 2)                        # /2
    y = b.conv_bn(y, w1, 3, 2)                        # /4
    y = _c2f(b, y, w1, depths[0], True)
    if upto == "stem":
        return done(y)
    y = b.conv_bn(y, w2, 3, 2)                        # /8
    p3 = _c2f(b, y, w2, depths[1], True)
    if upto == "p3":
        return done(p3)
    y = _down(b, p3, w3)                              # /16
    p4 = _c2f(b, y, w3, depths[2], True)
    if upto == "p4":
        return done(p4)
    y = _down(b, p4, w4)                              # /32
    y = _c2f(b, y, w4, depths[3], True)
    if upto == "c5":
        return done(y)
    y = _sppf(b, y)
    if upto == "sppf":
        return done(y)
    p5 = _psa(b, y)
    if upto == "psa":
        return done(p5)
    t = _c2f(b, b.concat([b.upsample2(p5), p4]), w3, 1, False)       # top-down /16
    if upto == "top":
        return done(t)
    s3 = _c2f(b, b.concat([b.upsample2(t), p3]), w2, 1, False)       # /8 out
    if upto == "s3":
        return done(s3)
    s4 = _c2f(b, b.concat([b.conv_bn(s3, w2, 3, 2), t]), w3, 1, False)   # /16 out
    if upto == "s4":
        return done(s4)
    s5 = _c2f(b, b.concat([_down(b, s4, w3), p5]), w4, 1, True)          # /32 out
    if upto == "s5":
        return done(s5)
    heads = [_head(b, s, nc=nc) for s in (s3, s4, s5)]
    return done(b.concat(heads, axis=2))


def yolo_input(batch: int, image: int = 640, seed: int = 4) -> np.ndarray:
    """U(0,1) NCHW images from ``default_rng(seed + 1)``."""
    return np.random.default_rng(seed + 1).uniform(0.0, 1.0, (batch, 3, image, image)).astype(np.float32)
