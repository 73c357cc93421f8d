"""CPU tests of the model semantics against the reference's own oracle formulations."""
import math

import torch

from faster_yoco_b200.config import build_args
from faster_yoco_b200.models.yoco import build_model
from faster_yoco_b200.ops import reference as ref


def test_param_count_matches_reference():
    assert build_args("yoco_3b").num_params() == 3_445_303_296


def test_state_dict_reference_names_roundtrip():
    args = build_args("yoco_tiny", max_seq_len=64)
    m = build_model(args)
    sd = m.state_dict()
    for k in ["self_decoder.layers.0.mixer.q_proj.weight", "self_decoder.layers.0.mixer.gt_proj.weight",
              "self_decoder.layers.1.ffn.fc1.weight", "self_decoder.layers.1.ffn.gate.weight",
              "cross_decoder.k_proj.weight", "cross_decoder.v_proj.weight", "cross_decoder.kv_layer_norm.weight",
              "cross_decoder.layers.0.mixer.q_proj.weight", "embed_tokens.weight", "output_projection.weight",
              "layer_norm.weight"]:
        assert k in sd, k
    assert sd["self_decoder.layers.0.mixer.gt_proj.weight"].shape == (4, 256)
    assert sum(v.numel() for v in sd.values()) == args.num_params()
    m2 = build_model(args)
    m2.load_state_dict(sd)
    for a, b in zip(m.parameters(), m2.parameters()):
        assert torch.equal(a, b)


def test_chunk_vs_parallel_vs_recurrent_retention():
    torch.manual_seed(0)
    B, H, L, D = 1, 2, 512, 32
    q = torch.randn(B, H, L, D, dtype=torch.float64)
    k = torch.randn(B, H, L, D, dtype=torch.float64)
    v = torch.randn(B, H, L, D, dtype=torch.float64)
    g = torch.nn.functional.logsigmoid(torch.randn(B, H, L, dtype=torch.float64)) / 16
    o_chunk = ref.chunk_gate_retention(q, k, v, g, chunk_size=128)
    o_par = ref.parallel_gate_retention(q, k, v, g)
    assert torch.allclose(o_chunk, o_par, atol=1e-5, rtol=1e-5)   # gates are cumsummed in fp32
    state = None
    outs = []
    for t in range(L):
        o, state = ref.recurrent_gate_retention(q[:, :, t:t + 1], k[:, :, t:t + 1].clone(), v[:, :, t:t + 1],
                                                g[:, :, t:t + 1], state)
        outs.append(o)
    assert torch.allclose(torch.cat(outs, 2), o_par, atol=1e-5, rtol=1e-5)


def test_rope_is_rotation_and_conjugate_inverts():
    x = torch.randn(2, 17, 3, 64)
    cos, sin = ref.rope_tables(64, 0, 17, 1e4, torch.float32)
    y = ref.apply_rope(x, cos, sin)
    assert torch.allclose(y.norm(dim=-1), x.norm(dim=-1), atol=1e-5)
    assert torch.allclose(ref.apply_rope(y, cos, sin, conjugate=True), x, atol=1e-5)


def test_rope_angles_use_linspace():
    a = ref.rope_angles(128, 3, 1e4)
    assert torch.allclose(a[1], 1.0 / (1e4 ** torch.linspace(0, 1, 64)))


def test_attention_oracle_window_and_gqa():
    torch.manual_seed(1)
    q = torch.randn(1, 40, 6, 16)
    k = torch.randn(1, 40, 2, 16)
    v = torch.randn(1, 40, 2, 16)
    o = ref.attention(q, k, v, causal=True, window=8)
    # row 20 attends to keys 13..20 only
    kk = k.repeat_interleave(3, dim=2)
    vv = v.repeat_interleave(3, dim=2)
    s = (q[0, 20, 0] @ kk[0, 13:21, 0].T) / 4.0
    exp = torch.softmax(s, -1) @ vv[0, 13:21, 0]
    assert torch.allclose(o[0, 20, 0], exp, atol=1e-5)


def test_forward_backward_tiny_and_incremental_decode_matches_full():
    torch.manual_seed(0)
    args = build_args("yoco_tiny", max_seq_len=512, max_batch_size=1)
    m = build_model(args).double().eval()
    x = torch.randint(0, 1024, (1, 300))
    with torch.no_grad():
        full, _ = m(x)
        st = {}
        pre, _ = m(x[:, :256], incremental_state=st, is_prefilling=True, start_pos=0)
        outs = [pre]
        for i in range(256, 300):
            o, _ = m(x[:, i:i + 1], incremental_state=st, is_prefilling=False, start_pos=i)
            outs.append(o)
        inc = torch.cat(outs, 1)
    assert torch.allclose(inc, full, atol=1e-7, rtol=1e-6), (inc - full).abs().max()


def test_sliding_window_model_decode_matches_full():
    torch.manual_seed(0)
    args = build_args("yoco_tiny", max_seq_len=256, max_batch_size=1, sliding_window=16)
    m = build_model(args).double().eval()
    x = torch.randint(0, 1024, (1, 60))
    with torch.no_grad():
        full, _ = m(x)
        st = {}
        pre, _ = m(x[:, :40], incremental_state=st, is_prefilling=True, start_pos=0)
        outs = [pre]
        for i in range(40, 60):
            o, _ = m(x[:, i:i + 1], incremental_state=st, is_prefilling=False, start_pos=i)
            outs.append(o)
    assert torch.allclose(torch.cat(outs, 1), full, atol=1e-7, rtol=1e-6)


def test_prefill_padding_path_matches_full():
    torch.manual_seed(0)
    args = build_args("yoco_tiny", max_seq_len=1024, max_batch_size=1)
    m = build_model(args).double().eval()
    x = torch.randint(0, 1024, (1, 700))
    with torch.no_grad():
        full, _ = m(x)
        st = {}
        a, _ = m(x[:, :300], incremental_state=st, is_prefilling=True, start_pos=0)       # padded to 512
        b, _ = m(x[:, 300:700], incremental_state=st, is_prefilling=True, start_pos=300)
    assert torch.allclose(torch.cat([a, b], 1), full, atol=1e-5, rtol=1e-5)   # fp32 gate sums
