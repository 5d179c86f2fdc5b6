"""The in-box PyTorch baseline (``bench.py --impl torch``) on CPU: decoding token by token through
the masked cache gives the same next tokens as prefilling the whole sequence."""
import torch

from hawking_b200.models.config import ModelConfig
from hawking_b200.utils.torch_baseline import TorchLlamaTP


def test_decode_matches_prefill():
    torch.manual_seed(0)
    cfg = ModelConfig(arch="llama", vocab=64, hidden=64, layers=2, n_heads=4, n_kv_heads=2, head_dim=16,
                      ffn=96, eps=1e-5, rope_theta=10000.0)
    m = TorchLlamaTP(cfg, 0, 1, "cpu", batch=1, capacity=24, seed=3)
    for L in m.layers:  # larger weights so the logits are far from ties
        for t in (L.wqkv, L.wo, L.wgu, L.wdown):
            t.mul_(20)
    m.lm_head.mul_(20)
    toks = torch.randint(0, cfg.vocab, (1, 12))
    ref = []
    for n in range(6, 12):  # next token after each prefix, by full prefill
        ref.append(int(m.prefill(toks[:, :n])[0]))
    m.prefill(toks[:, :5])
    got = []
    for n in range(5, 11):  # feed token n at position n, read the prediction for n + 1
        m.ids.fill_(int(toks[0, n]))
        m.pos.fill_(n)
        m._decode_eager()
        got.append(int(m.next_ids[0]))
    assert got == ref
