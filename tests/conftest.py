import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


@pytest.fixture(scope="session")
def bert_model():
    """BERT-base, random init from seed 0, eager masks, fp32 (CPU)."""
    import torch
    from transformers import BertConfig, BertModel
    torch.manual_seed(0)
    cfg = BertConfig(attn_implementation="eager")
    return BertModel(cfg).eval()


@pytest.fixture(scope="session")
def qwen3_model():
    """A small Qwen3 (3 layers, hidden 256, 4 Q heads, 2 KV heads, head_dim 128,
    QK-norm, RoPE theta 1e6), random init from seed 0, eager attention, fp32
    (CPU)."""
    import torch
    from transformers import Qwen3Config, Qwen3Model
    torch.manual_seed(0)
    cfg = Qwen3Config(vocab_size=1000, hidden_size=256, intermediate_size=512, num_hidden_layers=3,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=128,
                      max_position_embeddings=2048, rope_theta=1e6, tie_word_embeddings=False,
                      attn_implementation="eager")
    return Qwen3Model(cfg).eval()
