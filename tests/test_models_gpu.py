"""Model-level checks on the B200: the LLaMA baseline and the YOCO generation path on the native kernels versus
the PyTorch path of the same model in fp32."""
import pytest
import torch

from faster_yoco_b200 import ops

pytestmark = pytest.mark.gpu


def rel(x, ref):
    x, ref = x.float(), ref.float()
    return ((x - ref).abs().max() / ref.abs().max().clamp_min(1e-6)).item()


def test_llama_native_matches_fp32():
    from faster_yoco_b200.models.transformer import LLaMA, Transformer, llama_args_from_cfg
    torch.manual_seed(0)
    a = llama_args_from_cfg(256, 2, 2, 1, 1024, batch_size=2, tokens_per_sample=256)
    m32 = LLaMA(Transformer(a)).cuda()
    mbf = LLaMA(Transformer(a)).cuda()
    mbf.load_state_dict(m32.state_dict())
    mbf = mbf.to(torch.bfloat16)
    ids = torch.randint(0, 1024, (2, 256), device="cuda")
    ops.set_backend("torch")
    ref, _ = m32(ids)
    ref.pow(2).mean().backward()
    ops.set_backend("native")
    out, _ = mbf(ids)
    out.pow(2).mean().backward()
    assert rel(out, ref) < 3e-2
    g_ref = m32.model.layers[0].attention.wq.weight.grad
    g = mbf.model.layers[0].attention.wq.weight.grad
    assert rel(g, g_ref) < 6e-2


def test_yoco_generate_native():
    from faster_yoco_b200.config import build_args
    from faster_yoco_b200.data.tokenizers import ByteTokenizer
    from faster_yoco_b200.eval.generate import generate
    from faster_yoco_b200.models.yoco import YOCO
    torch.manual_seed(0)
    args = build_args("yoco_small", vocab_size=264, max_seq_len=1024, max_batch_size=1)
    with torch.device("cuda"):
        m = YOCO(args)
    m = m.to(torch.bfloat16).eval()
    ops.set_backend("native")
    tok = ByteTokenizer()
    prompt = torch.tensor([tok.encode("x" * 300, bos=True)], device="cuda")
    out = generate(m, prompt, tok, generate_tokens=4, chunk_length=128)
    assert out.shape == (1, prompt.shape[1] + 4) and torch.equal(out[:, :prompt.shape[1]], prompt)
