"""Expert blob format (the reference's experts_index.json) and model geometry.

One expert is one contiguous blob; blob (layer, expert) sits at
``(layer * n_experts + expert) * blob_bytes`` in the store (repack.py:141).
Inside a blob the components follow in the order gate_proj, up_proj,
down_proj, each as weight (U32 [out, in/8], eight 4-bit codes per word, low
nibble first), scales (BF16 [out, in/64]), biases (BF16 [out, in/64]) and,
for gpt-oss, bias (BF16 [out]) (repack.py:72-82, repack_gptoss.py:139-158).
The blob is padded to a whole number of 16 KiB pages (repack_gptoss.py:159).

The HBM slot arena uses the same layout, so a slot fill is one contiguous
copy and slot s of component c is at ``arena + s*blob_bytes + offset(c)``.
"""
import dataclasses
from dataclasses import dataclass, field

from . import _lib

PAGE = 16384
PROJS = ("gate_proj", "up_proj", "down_proj")
PARTS = ("weight", "scales", "biases", "bias")
# precision classes: component parts in ms_prec order
PREC_PARTS = ("weight", "scales", "biases", "bias", "scales_exp", "biases_exp")
CODE_BITS = (2, 3, 4, 8)
SCALE_FMTS = ("bf16", "fp8")


def code_row_bytes(n_in, bits):
    """Bytes of one row of codes: n_in*bits/8, rounded up to 16 (only 3-bit
    rows whose n_in is not a multiple of 128 carry padding)."""
    return -(-(n_in * bits // 8) // 16) * 16


@dataclass(frozen=True)
class Geometry:
    model: str                 # "qwen3" | "gptoss"
    d_model: int
    d_ff: int
    n_experts: int
    n_layers: int
    top_k: int
    group_size: int = 64
    bits: int = 4
    norm_topk_prob: bool = True
    scale_fmt: str = "bf16"
    components: tuple = field(default=(), compare=False)
    payload_bytes: int = 0
    blob_bytes: int = 0

    @property
    def proj_bias(self):
        return self.model == "gptoss"

    @property
    def n_keys(self):
        return self.n_layers * self.n_experts

    def comp(self, proj, part):
        for c in self.components:
            if c["proj"] == proj and c["part"] == part:
                return c
        raise KeyError(f"{proj}.{part}")

    def index(self):
        """experts_index.json content (repack.py:137-146)."""
        return dict(n_layers=self.n_layers, n_experts=self.n_experts, top_k=self.top_k,
                    blob_bytes=self.blob_bytes, payload_bytes=self.payload_bytes,
                    page_size=PAGE,
                    offset_formula="(layer * n_experts + expert) * blob_bytes",
                    quantization=dict(group_size=self.group_size, bits=self.bits),
                    components=[dict(c) for c in self.components])

    def to_c(self):
        g = _lib.MsGeom()
        g.model = _lib.MODEL_GPTOSS if self.model == "gptoss" else _lib.MODEL_QWEN3
        g.d_model, g.d_ff, g.n_experts = self.d_model, self.d_ff, self.n_experts
        g.n_layers, g.top_k = self.n_layers, self.top_k
        g.group_size, g.bits = self.group_size, self.bits
        g.norm_topk_prob = int(self.norm_topk_prob)
        g.proj_bias = int(self.proj_bias)
        g.blob_bytes = self.blob_bytes
        for i, proj in enumerate(PROJS):
            for j, part in enumerate(PARTS):
                try:
                    g.comp_offset[i][j] = self.comp(proj, part)["offset"]
                except KeyError:
                    g.comp_offset[i][j] = -1
        return g


def layout(d_model, d_ff, group_size=64, bits=4, proj_bias=False, scale_fmt="bf16"):
    """(components, payload_bytes, blob_bytes) for one expert. The default
    (4 bits, bf16) is the reference's layout; other precision classes keep
    the component order and add, for fp8 scales, the per-row exponents
    (scales_exp, biases_exp) after the biases. Offsets are 16-byte aligned."""
    fp8 = scale_fmt == "fp8"
    parts = ["weight", "scales", "biases"] + (["scales_exp", "biases_exp"] if fp8 else [])
    parts += ["bias"] if proj_bias else []
    comps, off = [], 0
    for proj in PROJS:
        n_out, n_in = (d_model, d_ff) if proj == "down_proj" else (d_ff, d_model)
        G = n_in // group_size
        for part in parts:
            if part == "weight":
                rb = code_row_bytes(n_in, bits)
                dt, shape, nb = "U32", [n_out, rb // 4], n_out * rb
            elif part == "bias":
                dt, shape, nb = "BF16", [n_out], n_out * 2
            elif part in ("scales_exp", "biases_exp"):
                dt, shape, nb = "U8", [n_out], n_out
            elif fp8:
                dt, shape, nb = "F8E4M3", [n_out, G], n_out * G
            else:
                dt, shape, nb = "BF16", [n_out, G], n_out * G * 2
            comps.append(dict(proj=proj, part=part, dtype=dt, shape=shape, offset=off, nbytes=nb))
            off += -(-nb // 16) * 16
    return tuple(comps), off, -(-off // PAGE) * PAGE


def precision(geom, bits, scale_fmt="bf16"):
    """The geometry of geom's experts stored as precision class (bits,
    scale_fmt): same shapes, that class's blob layout and size."""
    if bits not in CODE_BITS or scale_fmt not in SCALE_FMTS:
        raise ValueError(f"unsupported precision class ({bits}, {scale_fmt})")
    comps, payload, blob = layout(geom.d_model, geom.d_ff, geom.group_size, bits, geom.proj_bias,
                                  scale_fmt)
    return dataclasses.replace(geom, bits=bits, scale_fmt=scale_fmt, components=comps,
                               payload_bytes=payload, blob_bytes=blob)


def slot_geometry(base, classes):
    """The pool geometry for experts in `classes` (precision geometries of
    base): base's own 4-bit layout, with the slot and store stride of the
    largest class."""
    blob = max([base.blob_bytes] + [c.blob_bytes for c in classes])
    return dataclasses.replace(base, blob_bytes=blob)


def to_prec_c(cg):
    """ms_prec of a precision geometry (precision())."""
    p = _lib.MsPrec()
    p.bits = cg.bits
    p.scale_fmt = _lib.SCALE_FP8 if cg.scale_fmt == "fp8" else _lib.SCALE_BF16
    p.payload_bytes = -(-cg.payload_bytes // 16) * 16
    for i, proj in enumerate(PROJS):
        for j, part in enumerate(PREC_PARTS):
            try:
                p.comp_offset[i][j] = cg.comp(proj, part)["offset"]
            except KeyError:
                p.comp_offset[i][j] = -1
    return p


def make(model, d_model, d_ff, n_experts, n_layers, top_k, norm_topk_prob=True):
    comps, payload, blob = layout(d_model, d_ff, proj_bias=(model == "gptoss"))
    return Geometry(model=model, d_model=d_model, d_ff=d_ff, n_experts=n_experts,
                    n_layers=n_layers, top_k=top_k, norm_topk_prob=norm_topk_prob,
                    components=comps, payload_bytes=payload, blob_bytes=blob)


def qwen3(n_layers=48):
    """Qwen3-30B-A3B: 48 x 128 experts, top-8, d=2048, ff=768; blob 2,654,208 B
    = 162 pages (repack.py:13-14, kernels.py:58-63)."""
    return make("qwen3", 2048, 768, 128, n_layers, 8, True)


def gptoss(n_layers=36):
    """gpt-oss-120b: 36 x 128, top-4, d=ff=2880, projection biases; payload
    14,014,080 B padded to 14,024,704 B = 856 pages (HANDOFF table,
    scratchpad/stage_bench.py:11-12)."""
    return make("gptoss", 2880, 2880, 128, n_layers, 4, False)


def from_index(idx, model, d_model, d_ff, norm_topk_prob=True):
    """Geometry from a store's experts_index.json dict."""
    comps = tuple(sorted((dict(c) for c in idx["components"]), key=lambda c: c["offset"]))
    end = 0
    for c in comps:                      # engine_v3.py:168-178
        if c["offset"] != end:
            raise RuntimeError(f"blob layout has a hole before {c['proj']}.{c['part']}")
        end += c["nbytes"]
    if end > idx["blob_bytes"]:
        raise RuntimeError("components overrun the blob")
    return Geometry(model=model, d_model=d_model, d_ff=d_ff, n_experts=idx["n_experts"],
                    n_layers=idx.get("n_layers", 48), top_k=idx.get("top_k", 8),
                    group_size=idx["quantization"]["group_size"],
                    bits=idx["quantization"]["bits"], norm_topk_prob=norm_topk_prob,
                    components=comps, payload_bytes=end, blob_bytes=idx["blob_bytes"])
