"""Linear-layer shapes of the decoder stacks the SE12 path is measured on.

Each decoder layer has seven weight matrices (rows = out features,
cols = in features): q, k, v, o, gate, up, down; the LM head is
[vocab, hidden]. Shapes follow the benchmark configurations (Gemma-2 2B /
9B / 27B, Llama-3.1 70B).
"""

from __future__ import annotations

import dataclasses


@dataclasses.dataclass(frozen=True)
class DecoderShapes:
    name: str
    hidden: int
    q_out: int      # heads * head_dim
    kv_out: int     # kv heads * head_dim
    intermediate: int
    layers: int
    vocab: int

    def layer_matrices(self) -> list:
        """(name, rows, cols, input kind) of one decoder layer."""
        h, q, kv, i = self.hidden, self.q_out, self.kv_out, self.intermediate
        return [
            ("q_proj", q, h, "hidden"),
            ("k_proj", kv, h, "hidden"),
            ("v_proj", kv, h, "hidden"),
            ("o_proj", h, q, "attn"),
            ("gate_proj", i, h, "hidden"),
            ("up_proj", i, h, "hidden"),
            ("down_proj", h, i, "mlp"),
        ]

    # Projections that multiply the same input, computed as one segmented
    # matrix (one GEMV) when grouped: (group name, member names).
    GROUPS = (("qkv_proj", ("q_proj", "k_proj", "v_proj")), ("gate_up_proj", ("gate_proj", "up_proj")))

    def lm_head(self) -> tuple:
        return ("lm_head", self.vocab, self.hidden, "hidden")

    def input_width(self, kind: str) -> int:
        return {"hidden": self.hidden, "attn": self.q_out, "mlp": self.intermediate}[kind]

    @property
    def weights_per_layer(self) -> int:
        return sum(r * c for _, r, c, _ in self.layer_matrices())

    @property
    def total_weights(self) -> int:
        return self.layers * self.weights_per_layer + self.vocab * self.hidden


CONFIGS = {
    "gemma2-2b": DecoderShapes("gemma2-2b", hidden=2304, q_out=2048, kv_out=1024, intermediate=9216, layers=26, vocab=256000),
    "gemma2-9b": DecoderShapes("gemma2-9b", hidden=3584, q_out=4096, kv_out=2048, intermediate=14336, layers=42, vocab=256000),
    "gemma2-27b": DecoderShapes("gemma2-27b", hidden=4608, q_out=4096, kv_out=2048, intermediate=36864, layers=46, vocab=256000),
    "llama3.1-70b": DecoderShapes("llama3.1-70b", hidden=8192, q_out=8192, kv_out=1024, intermediate=28672, layers=80, vocab=128256),
}
