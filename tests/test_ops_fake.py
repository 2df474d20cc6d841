"""CPU: the shape / dtype rules (fake implementations) of every q3attn custom op, run on fake CUDA tensors. These are
what torch.compile traces through and what a captured frame allocates; no kernel runs."""
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import q3attn  # noqa: F401  (registers the ops)

OPS = torch.ops.q3attn
BF, F16 = torch.bfloat16, torch.float16


@pytest.fixture
def fake():
    with FakeTensorMode() as m:
        yield m


def e(*shape, dtype=BF):
    return torch.empty(*shape, dtype=dtype, device="cuda")


def i32(*shape):
    return torch.empty(*shape, dtype=torch.int32, device="cuda")


def i64(*shape):
    return torch.empty(*shape, dtype=torch.int64, device="cuda")


def test_decode_ops(fake):
    B, pages = 5, 40
    kc = e(pages, 16, 8, 128)
    seq, bt = i32(B), i32(B, 8)
    for out in (OPS.paged_decode(e(B, 16, 128), kc, kc, seq, bt, 0.1, 0),
                OPS.paged_decode_append(e(B, 16, 128), e(B, 8, 128), e(B, 8, 128), kc, kc, seq, bt, 0.1, 0),
                OPS.paged_decode_qkv(e(B, 4096), e(128), e(128), e(B, 128), e(B, 128), kc, kc, seq, bt, 0.1)):
        assert out.shape == (B, 16, 128) and out.dtype == BF and out.device.type == "cuda"


def test_code_predictor_ops(fake):
    B = 6
    K = e(B, 8, 16, 128)
    assert OPS.cp_attn(e(B, 16, 128), K, K, 4, 0.1).shape == (B, 2048)
    assert OPS.cp_step(e(B, 16, 128), e(B, 8, 128), e(B, 8, 128), K, K, 3, 0.1).shape == (B, 2048)
    assert OPS.cp_step_qkv(e(B, 4096), e(128), e(128), e(B, 128), e(B, 128), K, K, 3, 0.1).shape == (B, 2048)


def test_row_ops(fake):
    x = e(7, 1024)
    assert OPS.add_rms_norm(x, e(1024), e(7, 1024), 1e-6).shape == (7, 1024)
    assert OPS.silu_mul(e(7, 6144)).shape == (7, 3072)
    assert OPS.qk_norm_rope_(e(7, 4096), e(128), e(128), e(7, 128), e(7, 128)) is None


def test_prefill_and_append_ops(fake):
    T = 96
    q, k = e(T, 16, 128), e(T, 8, 128)
    cu = i32(3)
    assert OPS.prefill(q, k, k, cu, cu, 64, 0.1, True).shape == (T, 16, 128)
    kc = e(50, 16, 8, 128)
    assert OPS.prefill_paged(q, k, k, kc, kc, cu, cu, 64, i32(2), i32(2), i32(2, 10), 0.1, True, True).shape == \
        (T, 16, 128)
    assert OPS.kv_append_slots(k, k, kc, kc, i64(T)) is None
    assert OPS.kv_append_paged(k, k, kc, kc, i32(T), i32(T, 10), None) is None


def test_ring_and_sampler_ops(fake):
    B, n, H, hd = 4, 3, 16, 64
    q = e(B, n, H, hd, dtype=F16)
    ring = e(B + 1, 88, H, hd, dtype=F16)
    out = OPS.ring_window_attn(q, q, q, ring, ring, i64(B), i64(B), 71, 0.125, True)
    assert out.shape == (B, n, H * hd) and out.dtype == F16
    res = OPS.sample_topk(e(B, 3072, dtype=torch.float32), 0.9, 50, 7, i64(2), None, None, 1.0, None, None, 0, 0,
                          e(3072, 1024))
    ids, emb = res
    assert ids.shape == (B,) and ids.dtype == torch.int64
    assert emb.shape == (B, 1024) and emb.dtype == BF


def test_ops_trace_as_single_opaque_nodes():
    """Traced with fake tensors (as torch.compile's front end does), each op is one node of the graph, mutating ones
    included: nothing of the attention is decomposed into aten ops."""
    from torch.fx.experimental.proxy_tensor import make_fx

    def layer(q, k, v, kc, vc, seq, bt, cq, K):
        o = OPS.paged_decode_append(q, k, v, kc, vc, seq, bt, 0.1, 0)
        c = OPS.cp_step(cq, k, v, K, K, 2, 0.1)
        return o.float().sum() + c.float().sum()

    with FakeTensorMode():
        args = (e(3, 16, 128), e(3, 8, 128), e(3, 8, 128), e(20, 16, 8, 128), e(20, 16, 8, 128), i32(3), i32(3, 4),
                e(3, 16, 128), e(3, 8, 16, 128))
        g = make_fx(layer, tracing_mode="fake")(*args)
    targets = [str(n.target) for n in g.graph.nodes if n.op == "call_function"]
    assert targets.count("q3attn.paged_decode_append.default") == 1
    assert targets.count("q3attn.cp_step.default") == 1
    assert not any("softmax" in t or "bmm" in t or "matmul" in t for t in targets)
