"""Drop-in token embedding: nn.Embedding whose forward is the B200 gather kernel.

Devstral2Model builds ``self.embed_tokens = nn.Embedding(vocab_size, hidden_size)`` and calls
``self.embed_tokens(input_ids)`` (miniagentserve/models/devstral2/devstral2.py:260, :282). This class
subclasses nn.Embedding, so construction, initialisation, the ``weight`` parameter, the state-dict key
(``model.embed_tokens.weight``, devstral2.py:386-387) and weight tying with the LM head
(devstral2.py:317-318) are unchanged; only forward runs the CUDA gather (ops.embedding).

Inference only, like the reference's serving path (it runs under torch.inference_mode): the gather has
no backward, and the options that only shape training (max_norm, sparse) are rejected.
"""
from __future__ import annotations

import torch
from torch import nn

from . import ops

__all__ = ["Embedding"]


class Embedding(nn.Embedding):
    def forward(self, input: torch.Tensor) -> torch.Tensor:
        if self.max_norm is not None:
            raise NotImplementedError("mas_b200 Embedding: max_norm renormalisation is not supported")
        if self.sparse:
            raise NotImplementedError("mas_b200 Embedding: sparse gradients are not supported")
        return ops.embedding(input, self.weight)
