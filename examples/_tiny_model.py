"""The randomly initialised one-layer Qwen3 model both examples train.

On a GPU the model runs in bf16 through this package's sm_100a kernels (whose
attention takes head dims 64 and 128); on a CPU it runs in fp32 through the
plain torch reference ops.
"""

import torch

from thundersync_b200 import Qwen3Config, Qwen3ForCausalLM

# Token ids below this bound are valid inputs; the examples' prompts and turns
# are arbitrary ids in this range rather than tokenized text.
VOCAB_SIZE = 64


def tiny_qwen3(device: torch.device) -> torch.nn.Module:
    cfg = Qwen3Config(vocab_size=VOCAB_SIZE, hidden_size=128, intermediate_size=256, num_hidden_layers=1,
                      num_attention_heads=2, num_key_value_heads=1, head_dim=64, max_position_embeddings=128,
                      tie_word_embeddings=False)
    with torch.device(device):
        model = Qwen3ForCausalLM(cfg)
    return model.to(torch.bfloat16 if device.type == "cuda" else torch.float32)
