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
