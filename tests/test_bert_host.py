"""Host-side logic of the BERT drop-in (no GPU): the module swap keeps the
model's train / eval mode, and the encoder loop compacts a layer's tail only
where that is row-for-row the reference's computation."""
import pytest
import torch
from transformers import BertConfig, BertModel

from spatten_b200.bert import _compactable, patch_bert


def _model(layers=2, dtype=torch.float16):
    torch.manual_seed(0)
    cfg = BertConfig(num_hidden_layers=layers, attn_implementation="sdpa")
    return BertModel(cfg).to(dtype)


def test_patch_keeps_eval_and_train_mode():
    m = patch_bert(_model().eval(), enable_token_prune=True, token_keep_ratio=0.9)
    assert all(not layer.attention.self.training for layer in m.encoder.layer)
    m = patch_bert(_model().train(), enable_token_prune=True, token_keep_ratio=0.9)
    assert all(layer.attention.self.training for layer in m.encoder.layer)


def test_compactable_conditions():
    m = patch_bert(_model().eval(), enable_token_prune=True, token_keep_ratio=0.9)
    layer = m.encoder.layer[0]
    attn = layer.attention.self
    h = torch.zeros(2, 8, 768, dtype=torch.float16)
    assert not _compactable(layer, attn, h, last=False)        # a CPU tensor: no kernel to run


@pytest.mark.gpu
def test_compactable_conditions_on_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    m = patch_bert(_model().cuda().eval(), enable_token_prune=True, token_keep_ratio=0.9)
    layer = m.encoder.layer[0]
    attn = layer.attention.self
    h = torch.zeros(2, 8, 768, dtype=torch.float16, device="cuda")
    assert _compactable(layer, attn, h, last=False)
    assert not _compactable(layer, attn, h, last=True)     # the last layer's rows are the output
    attn.compact_ffn = False
    assert not _compactable(layer, attn, h, last=False)
    attn.compact_ffn = True
    attn.train()                                           # dropout in the tail: not row-for-row
    assert not _compactable(layer, attn, h, last=False)
    attn.eval()
    assert not _compactable(layer, attn, h.float(), last=False)
    attn.enable_token_prune = False
    assert not _compactable(layer, attn, h, last=False)
