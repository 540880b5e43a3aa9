"""CPU: the drop-in module keeps the reference's constructor contract and
fails loudly (no CPU fallback) instead of computing on the host."""
import pytest
import torch


def test_constructor_matches_reference_contract(esa):
    m = esa.ElasticSparseAttention(layer_idx=2, num_hidden_layers=8, num_attention_heads=32,
                                   head_dim=128, attention_length=64, max_seq_len=4096,
                                   num_key_value_heads=8)
    assert m.num_kv_groups == 4
    assert m.scaling == 128 ** -0.5
    assert m.implementation == "triton"
    assert m.num_key_value_heads == 8
    m2 = esa.ElasticSparseAttention(0, 1, 4, 64, 16, 128)
    assert m2.num_key_value_heads == 4 and m2.num_kv_groups == 1
    for impl in ("triton", "naive", "dense"):
        assert esa.ElasticSparseAttention(0, 4, 4, 64, 16, 128, implementation=impl).implementation == impl
    # state_dict stays empty: the pattern is not a persistent buffer (reference :466-468)
    assert len(m.state_dict()) == 0


def test_constructor_errors(esa):
    with pytest.raises(ValueError, match="Invalid implementation 'flash'"):
        esa.ElasticSparseAttention(0, 4, 4, 64, 16, 128, implementation="flash")
    with pytest.raises(ValueError, match="must be divisible by"):
        esa.ElasticSparseAttention(0, 4, 6, 64, 16, 128, num_key_value_heads=4)


def test_forward_length_check_and_no_cpu_path(esa):
    m = esa.ElasticSparseAttention(0, 4, 2, 32, 16, 64)
    q = torch.randn(1, 2, 8, 32)
    k = torch.randn(1, 2, 65, 32)
    with pytest.raises(ValueError, match="exceeds the maximum length"):
        m(q, k, k)
    k = torch.randn(1, 2, 8, 32)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        m(q, k, k)


def test_q_longer_than_kv_needs_cache_position(esa):
    m = esa.ElasticSparseAttention(0, 4, 2, 32, 16, 64)
    with pytest.raises(ValueError, match="needs cache_position"):
        m(torch.randn(1, 2, 9, 32), torch.randn(1, 2, 8, 32), torch.randn(1, 2, 8, 32))


def test_pattern_spec(esa):
    s = esa.PatternSpec(3, 8, 64)
    assert (s.layer_idx, s.num_hidden_layers, s.attention_length) == (3, 8, 64)


def test_prepare_rows_host_checks(esa):
    """cache_position on the host: negative entries wrap (torch indexing of the
    reference's [:kv_len] slice), out-of-range entries raise IndexError, a
    wrong count raises ValueError -- all without a GPU."""
    prep = esa.ElasticSparseAttention._prepare_rows
    rows = prep(torch.tensor([5, -1, 0]), 3, 10, "cpu")
    assert rows.tolist() == [5, 9, 0] and rows.dtype == torch.int64
    assert prep([3, 4], 2, 10, "cpu").tolist() == [3, 4]
    with pytest.raises(IndexError):
        prep(torch.tensor([10]), 1, 10, "cpu")
    with pytest.raises(IndexError):
        prep(torch.tensor([-11]), 1, 10, "cpu")
    with pytest.raises(ValueError):
        prep(torch.tensor([1, 2]), 3, 10, "cpu")


def test_decoder_stack_builds_on_cpu(esa):
    """The C4 harness module: parameter shapes, initialisation and the GEMM
    FLOP count (its kernels need a GPU; construction does not)."""
    m = esa.ElasticDecoderStack(vocab_size=100, hidden_size=64, num_hidden_layers=2,
                                num_attention_heads=4, num_key_value_heads=2,
                                intermediate_size=96, attention_length=8, max_seq_len=32,
                                dtype=torch.float32, device="cpu")
    shapes = {n: tuple(p.shape) for n, p in m.named_parameters()}
    assert shapes["layers.0.qkv_proj"] == ((4 + 2 * 2) * 16, 64)
    assert shapes["layers.1.gate_up_proj"] == (2 * 96, 64)
    assert shapes["lm_head"] == (100, 64)
    assert torch.equal(m.final_norm, torch.ones(64))
    assert 0.015 < m.embed.std().item() < 0.025
    assert [s.layer_idx for s in m.specs] == [0, 1] and m.specs[0].num_hidden_layers == 2
    per_layer = 64 * 128 + 64 * 64 + 3 * 64 * 96
    assert m.flops_per_token(32) == 6.0 * (2 * per_layer + 100 * 64)
    inv = esa.layer_ops.rope_inv_freq(16, 10000.0, "cpu")
    assert torch.allclose(inv, 1.0 / 10000.0 ** (torch.arange(0, 16, 2).float() / 16))
    with pytest.raises(ValueError):
        esa.ElasticDecoderStack(hidden_size=64, num_attention_heads=4, num_key_value_heads=3,
                                vocab_size=10, intermediate_size=8, dtype=torch.float32,
                                device="cpu")


def test_head_share_splits_whole_groups(esa):
    """C3's head split: rank r of N holds Hkv / N whole GQA groups."""
    shares = [esa.head_share(32, 8, r, 4) for r in range(4)]
    assert shares == [(0, 8, 0, 2), (8, 8, 2, 2), (16, 8, 4, 2), (24, 8, 6, 2)]
    assert esa.head_share(16, 16, 7, 8) == (14, 2, 14, 2)
    with pytest.raises(ValueError, match="whole GQA groups"):
        esa.head_share(32, 8, 0, 3)
    with pytest.raises(ValueError, match="outside"):
        esa.head_share(32, 8, 4, 4)
    m = esa.HeadShardedElasticSparseAttention(3, 8, 32, 128, 64, 4096, num_key_value_heads=8,
                                              rank=1, world_size=4)
    assert m.pattern.head_offset == 8 and m.pattern.pattern_heads == 32
    with pytest.raises(ValueError, match="holds 8 query / 2 KV heads"):
        m(torch.randn(1, 4, 8, 128), torch.randn(1, 2, 8, 128), torch.randn(1, 2, 8, 128))
