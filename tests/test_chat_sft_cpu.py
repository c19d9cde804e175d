"""Chat SFT of a tiny Qwen3 policy on CPU: assistant-only packing, the masked loss falls, and the
trained model answers the held-out prompt with the trained turn and its end marker."""

import torch

from marin_experiments_b200.data.chat import IM_END
from marin_experiments_b200.data.tokenize import ByteTokenizer
from marin_experiments_b200.models.qwen3 import Qwen3Config, Qwen3Model
from marin_experiments_b200.rl.chat_sft import ChatSFTConfig, pack_conversations, run_chat_sft


def _model():
    cfg = Qwen3Config(vocab_size=257, hidden_dim=64, intermediate_dim=128, num_layers=2, num_heads=2, num_kv_heads=1,
                      head_dim=32, max_seq_len=128)
    return Qwen3Model(cfg).init_weights(seed=0)


CONVS = [[{"role": "user", "content": "hi"}, {"role": "assistant", "content": "ok"}],
         [{"role": "system", "content": "be brief"}, {"role": "user", "content": "hi"},
          {"role": "assistant", "content": "ok"}]]


def test_packing_masks_assistant_turns_only():
    tok = ByteTokenizer()
    t, m = pack_conversations(CONVS, tok, 32)
    assert t.shape[1] == 32 and t.shape == m.shape
    text = bytes(int(x) for x, w in zip(t.view(-1), m.view(-1)) if w > 0 and x < 256).decode()
    assert text == "ok" + IM_END + "\n" + "ok" + IM_END + "\n"


def test_chat_sft_learns_the_turn():
    torch.manual_seed(0)
    tok = ByteTokenizer()
    model = _model()
    cfg = ChatSFTConfig(steps=120, batch_size=4, lr=3e-3, max_seq_len=64, eval_tokens=16, seed=0)
    out = run_chat_sft(model, tok, CONVS * 8, cfg, eval_prompts=["hi"])
    assert out["losses"][-1] < 0.2 * out["losses"][0]
    assert out["after"][0] == "ok" + IM_END
    assert out["before"][0] != out["after"][0]
