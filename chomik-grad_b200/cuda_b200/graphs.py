"""Host-side helpers around the reference's Llama graphs.

The plugin compiles the graphs that ``chomikgrad.llama`` builds (the reference
package itself, unmodified).  What the reference package lacks, and the
plugin's runtimes need, lives here:

* ``decode_masks``: the per-step additive attention mask and cache write mask
  that the generation loop builds (generate_tinyllama.py:781-786, an example
  script outside the package);
* ``rope_angles``: the float32 angle table ``pos * theta^(-2j/hd)`` formed the
  way ``_rope_rotations`` forms it (chomikgrad/llama.py:135-140), from which
  the planner derives the RoPE cos/sin tables when a graph carries no
  rotation constant;
* ``GraphHelpers``: two building blocks (token embedding, attention with the
  ``sdpa`` lowering hint over un-repeated K/V) for the plugin's own graph
  builders -- the batched decode step and the tensor-parallel shards -- which
  subclass the reference's ``LlamaDecoderStep`` / ``LlamaForCausalLM``.
"""

from __future__ import annotations

from typing import Tuple

import numpy as np

from chomikgrad.llama import _prefer_lowering
from chomikgrad.tensor import Tensor

# The additive mask value of the reference's causal and decode masks (llama.py:250-258).
MASKED = -1e4


def decode_masks(position: int, context: int, dtype: np.dtype) -> Tuple[np.ndarray, np.ndarray]:
    """(1, 1, 1, ctx) attention mask (0 up to ``position``, -1e4 after) and (1, 1, ctx, 1) write mask."""
    attention = np.full((1, 1, 1, context), MASKED, dtype=dtype)
    attention[..., : position + 1] = 0
    write = np.zeros((1, 1, context, 1), dtype=dtype)
    write[:, :, position, :] = 1
    return attention, write


def rope_angles(positions: int, head_size: int, theta: float, offset: int = 0) -> np.ndarray:
    """(positions, hd/2) float32 angles, every operation in float32 as llama.py:135-140."""
    where = np.arange(offset, offset + positions, dtype=np.float32)
    inverse = 1.0 / (theta ** (np.arange(0, head_size, 2, dtype=np.float32) / head_size))
    return where[:, None] * inverse[None, :]


class GraphHelpers:
    """Mixed into subclasses of the reference's Llama classes (needs ``weights``, ``config``,
    ``_repeat_kv``)."""

    def _embed(self, token_matrix: Tensor) -> Tensor:
        """Token ids -> rows of the embedding table (llama.py:398-401)."""
        table = self.weights["model.embed_tokens.weight"]
        if len(token_matrix.shape) == 2:
            return table.gather(token_matrix)
        return token_matrix @ table

    def _attend(self, query: Tensor, keys: Tensor, values: Tensor, mask: Tensor) -> Tensor:
        """Masked softmax attention over the GQA-broadcast K/V, hinted ``sdpa`` over the
        un-broadcast K/V (the decode form of llama.py:514-525)."""
        scale = np.sqrt(self.config.head_size)
        scores = (query @ self._repeat_kv(keys).transpose(-2, -1)) / scale + mask
        attended = scores.softmax(axis=-1) @ self._repeat_kv(values)
        return _prefer_lowering(attended, "sdpa", (query, keys, values, mask), 1 / scale)
