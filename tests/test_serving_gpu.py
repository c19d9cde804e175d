"""Qwen3 serving path on the GPU (fused qkv GEMM, head RMSNorm+RoPE kernel, KV-cache append,
tcgen05 prefill attention, split-K decode attention, CUDA-graph decode) against the fp32 oracle."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("hd,heads,kv,graphs", [(64, 4, 2, True), (128, 2, 2, False)])
def test_prefill_and_decode_match_reference(hd, heads, kv, graphs):
    from marin_experiments_b200.data.tokenize import ByteTokenizer
    from marin_experiments_b200.models.qwen3 import Qwen3Config, Qwen3Model
    from marin_experiments_b200.ops._ext import check_kernel_errors
    from marin_experiments_b200.serving.engine import Engine

    cfg = Qwen3Config(vocab_size=512, hidden_dim=256, intermediate_dim=256, num_layers=2, num_heads=heads,
                      num_kv_heads=kv, head_dim=hd, rope_theta=10000.0, max_seq_len=512)
    ref = Qwen3Model(cfg).init_weights(3)
    gpu = Qwen3Model(cfg)
    gpu.load_state_dict(ref.state_dict())
    gpu = gpu.cuda()
    eng = Engine(gpu, ByteTokenizer(), max_batch=2, max_len=512, use_graphs=graphs)
    g = torch.Generator().manual_seed(0)
    p0 = torch.randint(0, 512, (37,), generator=g).tolist()
    p1 = torch.randint(0, 512, (50,), generator=g).tolist()
    l0 = eng._prefill(p0, 0)
    l1 = eng._prefill(p1, 1)
    r0 = ref.forward_reference(torch.tensor([p0]))[:, -1]
    r1 = ref.forward_reference(torch.tensor([p1]))[:, -1]
    assert rel(l0.cpu(), r0) < 3e-2 and rel(l1.cpu(), r1) < 3e-2
    seqs = [list(p0), list(p1)]
    pos = torch.tensor([len(p0), len(p1)], dtype=torch.int32, device="cuda")
    for step in range(4):
        nxt = torch.randint(0, 512, (2,), generator=g)
        out = eng._decode(nxt.cuda(), pos)
        for j in range(2):
            seqs[j].append(int(nxt[j]))
            want = ref.forward_reference(torch.tensor([seqs[j]]))[:, -1]
            assert rel(out[j:j + 1].cpu(), want) < 3e-2, (step, j)
        pos = pos + 1
    torch.cuda.synchronize()
    check_kernel_errors()


def test_generate_on_gpu():
    from marin_experiments_b200.serving.server import tiny_engine

    eng = tiny_engine("cuda")
    a = eng.generate(["hello", "world"], max_tokens=12, temperature=0.0)
    b = eng.generate(["hello", "world"], max_tokens=12, temperature=0.0)
    assert a == b and all(isinstance(x, str) for x in a)


def test_refresh_weights_in_place():
    """After the policy's weights change, ``refresh_weights`` makes the engine (and its captured decode
    graph) sample exactly what a freshly built engine over the new weights samples."""
    from marin_experiments_b200.data.tokenize import ByteTokenizer
    from marin_experiments_b200.models.qwen3 import Qwen3Config, Qwen3Model
    from marin_experiments_b200.serving.engine import Engine, SamplingParams

    cfg = Qwen3Config(vocab_size=512, hidden_dim=256, intermediate_dim=256, num_layers=2, num_heads=4,
                      num_kv_heads=2, head_dim=64, rope_theta=10000.0, max_seq_len=256)
    m = Qwen3Model(cfg).init_weights(5).cuda()
    tok = ByteTokenizer()
    eng = Engine(m, tok, max_batch=2, max_len=256)
    p = SamplingParams(max_tokens=10, temperature=0.0)
    prompts = [tok.encode("alpha"), tok.encode("beta gamma")]
    first = eng.generate_ids(prompts, p)
    with torch.no_grad():
        for L in m.layers:
            L.w_o.mul_(-1.5)
            L.w_down.add_(0.05 * torch.randn_like(L.w_down))
        m.embed.mul_(1.3)
    eng.refresh_weights()
    again = eng.generate_ids(prompts, p)
    fresh = Engine(m, tok, max_batch=2, max_len=256).generate_ids(prompts, p)
    assert again == fresh and again != first
