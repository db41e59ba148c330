"""PARAM-001 tensor table: the flat order, shapes and decay groups.

Restates ``GqaDimensions::parameter_layout`` (src/train/full_state.rs:113-154)
and ``parameter_specs`` (src/model/oracle.rs:177-275), with decay membership
``weight_decay_for`` (src/train/full_state.rs:179-181).  The two model files
the reference ships are embedded as presets (model-135m.example.json,
model-smoke.example.json) so nothing has to be read from the reference tree.

The reference's layout cannot express tied embeddings; for
model-smoke.example.json (``tie_embeddings: true``) this table drops
``lm_head.weight`` -- 20 tensors, 4,489,856 parameters -- and says so.
"""
from __future__ import annotations

import hashlib
import struct
from dataclasses import dataclass

import numpy as np

# src/model.rs:10-11
CANONICAL_PARAMETER_COUNT = 135_285_504
REFERENCE_PARAMETER_COUNT = 124_668_672


def weight_decay_for(name: str) -> bool:
    """src/train/full_state.rs:179-181: exactly the RMSNorm scales are no-decay."""
    return not name.endswith("norm.weight")


@dataclass(frozen=True)
class GqaDimensions:
    vocabulary: int
    width: int
    ffn_width: int
    layers: int
    query_heads: int
    key_value_heads: int
    head_width: int
    tie_embeddings: bool = False

    @staticmethod
    def canonical() -> "GqaDimensions":
        """src/train/full_state.rs:57-68 (= model-135m.example.json)."""
        return GqaDimensions(32_000, 768, 2_432, 12, 12, 4, 64, False)

    @staticmethod
    def reference_124m() -> "GqaDimensions":
        """src/model/oracle.rs:107-123 (gqa-124m-ref-v1, FFN 2,048)."""
        return GqaDimensions(32_000, 768, 2_048, 12, 12, 4, 64, False)

    @staticmethod
    def smoke() -> "GqaDimensions":
        """model-smoke.example.json: d_model 128, d_ff 384, 2 layers, 4/2 heads, tied."""
        return GqaDimensions.from_model_json(
            {"vocab_size": 32000, "d_model": 128, "d_ff": 384, "n_layers": 2, "n_heads": 4,
             "n_kv_heads": 2, "tie_embeddings": True})

    @staticmethod
    def oracle_fixture() -> "GqaDimensions":
        """src/train/full_state.rs:74-85: the 140-parameter P9B fixture shape."""
        return GqaDimensions(4, 4, 4, 1, 2, 1, 2, False)

    @staticmethod
    def from_model_json(cfg: dict) -> "GqaDimensions":
        heads = int(cfg["n_heads"])
        width = int(cfg["d_model"])
        if width % heads:
            raise ValueError("d_model must be a multiple of n_heads")
        return GqaDimensions(
            vocabulary=int(cfg["vocab_size"]),
            width=width,
            ffn_width=int(cfg["d_ff"]),
            layers=int(cfg["n_layers"]),
            query_heads=heads,
            key_value_heads=int(cfg["n_kv_heads"]),
            head_width=width // heads,
            tie_embeddings=bool(cfg.get("tie_embeddings", False)),
        )

    def validate(self) -> None:
        """src/train/full_state.rs:87-107."""
        if (min(self.vocabulary, self.width, self.ffn_width, self.layers, self.query_heads,
                self.key_value_heads, self.head_width) <= 0
                or self.head_width % 2
                or self.query_heads * self.head_width != self.width
                or self.query_heads % self.key_value_heads):
            raise ValueError("E1_DIMENSIONS_INVALID: not a valid untied pre-norm GQA shape")

    @property
    def key_value_width(self) -> int:
        return self.key_value_heads * self.head_width

    def parameter_layout(self) -> list[tuple[str, tuple[int, ...]]]:
        """The stable PARAM-001 order (src/train/full_state.rs:113-154)."""
        self.validate()
        out: list[tuple[str, tuple[int, ...]]] = [
            ("tok_embeddings.weight", (self.vocabulary, self.width))]
        for b in range(self.layers):
            out.append((f"blocks.{b}.attn_norm.weight", (self.width,)))
            out.append((f"blocks.{b}.attn.q.weight", (self.width, self.width)))
            for proj in ("k", "v"):
                out.append((f"blocks.{b}.attn.{proj}.weight", (self.key_value_width, self.width)))
            out.append((f"blocks.{b}.attn.o.weight", (self.width, self.width)))
            out.append((f"blocks.{b}.ffn_norm.weight", (self.width,)))
            for proj in ("gate", "up"):
                out.append((f"blocks.{b}.ffn.{proj}.weight", (self.ffn_width, self.width)))
            out.append((f"blocks.{b}.ffn.down.weight", (self.width, self.ffn_width)))
        out.append(("final_norm.weight", (self.width,)))
        if not self.tie_embeddings:
            out.append(("lm_head.weight", (self.vocabulary, self.width)))
        return out

    def parameter_count(self) -> int:
        return sum(int(np.prod(shape)) for _, shape in self.parameter_layout())


@dataclass(frozen=True)
class TensorTable:
    """The device-side tensor table: names, element counts, decay flags and
    the flat offsets of each tensor in the PARAM-001 buffer."""

    names: tuple[str, ...]
    shapes: tuple[tuple[int, ...], ...]
    elements: tuple[int, ...]
    decay: tuple[bool, ...]

    @property
    def offsets(self) -> np.ndarray:
        off = np.zeros(len(self.elements) + 1, dtype=np.uint64)
        off[1:] = np.cumsum(np.asarray(self.elements, dtype=np.uint64))
        return off

    @property
    def parameter_count(self) -> int:
        return int(sum(self.elements))

    def __len__(self) -> int:
        return len(self.names)

    @staticmethod
    def from_dimensions(dims: GqaDimensions) -> "TensorTable":
        layout = dims.parameter_layout()
        return TensorTable(
            names=tuple(n for n, _ in layout),
            shapes=tuple(s for _, s in layout),
            elements=tuple(int(np.prod(s)) for _, s in layout),
            decay=tuple(weight_decay_for(n) for n, _ in layout),
        )

    @staticmethod
    def from_sizes(sizes, decay=None, prefix: str = "t") -> "TensorTable":
        """An arbitrary table (tests: odd sizes, boundaries inside vectors)."""
        sizes = [int(s) for s in sizes]
        if decay is None:
            decay = [True] * len(sizes)
        return TensorTable(
            names=tuple(f"{prefix}{i}.weight" for i in range(len(sizes))),
            shapes=tuple((s,) for s in sizes),
            elements=tuple(sizes),
            decay=tuple(bool(d) for d in decay),
        )

    def layout_sha256(self) -> str:
        """src/model/oracle.rs:1287-1307 parameter_layout_sha256 over the specs
        (initialisation byte: Ones for the norm scales, Normal otherwise)."""
        h = hashlib.sha256()
        h.update(b"python-slm/parameter-layout/v1\0")
        for name, shape, n, dec in zip(self.names, self.shapes, self.elements, self.decay):
            raw = name.encode()
            h.update(struct.pack("<Q", len(raw)) + raw)
            h.update(struct.pack("<Q", len(shape)))
            for d in shape:
                h.update(struct.pack("<Q", d))
            h.update(struct.pack("<Q", n))
            h.update(bytes([1 if name.endswith("norm.weight") else 0]))
            h.update(bytes([0 if dec else 1]))
        return h.hexdigest()
