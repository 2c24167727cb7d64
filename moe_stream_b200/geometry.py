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
from dataclasses import dataclass, field

from . import _lib

PAGE = 16384
PROJS = ("gate_proj", "up_proj", "down_proj")
PARTS = ("weight", "scales", "biases", "bias")


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


def layout(d_model, d_ff, group_size=64, bits=4, proj_bias=False):
    """(components, payload_bytes, blob_bytes) for one expert."""
    parts = PARTS if proj_bias else PARTS[:3]
    comps, off = [], 0
    for proj in PROJS:
        n_out, n_in = (d_model, d_ff) if proj == "down_proj" else (d_ff, d_model)
        for part in parts:
            if part == "weight":
                dt, shape, nb = "U32", [n_out, n_in * bits // 32], n_out * n_in * bits // 8
            elif part == "bias":
                dt, shape, nb = "BF16", [n_out], n_out * 2
            else:
                dt, shape, nb = "BF16", [n_out, n_in // group_size], n_out * (n_in // group_size) * 2
            comps.append(dict(proj=proj, part=part, dtype=dt, shape=shape, offset=off, nbytes=nb))
            off += nb
    return tuple(comps), off, -(-off // PAGE) * PAGE


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
