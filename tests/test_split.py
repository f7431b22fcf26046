"""Tensor-parallel split rules (cpq_tp_split_state), CPU only.

The first seven tests restate the reference's own unit tests of
crates/codpiece-model/src/split.rs:364-532 (same fixture, same assertions)
against the C++ restatement in libcpq; the rest cover the benchmark's
27B-shaped stack at 2/4/8 devices.
"""
import pytest

from codpiece_b200 import tp

HP = tp.HP_QWEN35_27B


def key_dim():
    return HP.d_state * HP.n_k_heads


def conv_dim():
    return 2 * key_dim() + HP.d_inner


def extent(st, n=2):
    return sum(sum(st.ne[s * n:(s + 1) * n]) * st.nr[s] for s in range(st.n_segments))


def test_qwen35_head_ratio_segments_cover_the_tensor():  # split.rs:364-389
    assert key_dim() == 2048 and conv_dim() == 10240
    for n, e in (("blk.0.attn_qkv.weight", conv_dim()), ("blk.0.ssm_conv1d.weight", conv_dim()),
                 ("blk.0.attn_gate.weight", HP.d_inner), ("blk.0.ssm_out.weight", HP.d_inner),
                 ("blk.0.ssm_a", HP.n_v_heads), ("blk.0.ssm_dt.bias", HP.n_v_heads),
                 ("blk.0.ssm_alpha.weight", HP.n_v_heads)):
        st = tp.split_state(n, HP, e, 32, 2)
        assert st.axis in (tp.AXIS_0, tp.AXIS_1), n
        assert extent(st) == e, n


def test_lm_head_is_replicated_to_keep_sampling_in_graph():  # split.rs:391-396
    assert tp.split_state("output.weight", HP, 248320, 32, 2).axis == tp.MIRRORED


def test_split_axes_match_llama_cpp():  # split.rs:398-424
    ax = lambda n: tp.split_state(n, HP, 1024, 32, 2).axis  # noqa: E731
    assert ax("blk.3.attn_q.weight") == tp.AXIS_1
    assert ax("blk.3.attn_output.weight") == tp.AXIS_0
    assert ax("blk.0.ffn_up.weight") == tp.AXIS_1
    assert ax("blk.0.ffn_gate.weight") == tp.AXIS_1
    assert ax("blk.0.ffn_down.weight") == tp.AXIS_0
    assert ax("blk.0.ssm_out.weight") == tp.AXIS_0
    assert ax("output.weight") == tp.MIRRORED
    for n in ("token_embd.weight", "output_norm.weight", "blk.0.attn_norm.weight",
              "blk.0.post_attention_norm.weight", "blk.0.ssm_norm.weight", "blk.3.attn_q_norm.weight"):
        assert ax(n) == tp.MIRRORED, n


def test_session_caches_classified():  # split.rs:426-439
    assert tp.split_state("cache_k_l3", HP, 1024, 32, 2).axis == tp.AXIS_0
    assert tp.split_state("cache_v_l3", HP, 1024, 32, 2).axis == tp.AXIS_0
    conv = tp.split_state("cache_conv_l0", HP, conv_dim(), 32, 2)
    assert conv.axis == tp.AXIS_1 and extent(conv) == conv_dim()
    gdn = tp.split_state("cache_gdn_l0", HP, HP.n_v_heads, 32, 2)
    assert gdn.axis == tp.AXIS_2 and extent(gdn) == HP.n_v_heads


CASES = [("blk.0.attn_qkv.weight", 10240, 32), ("blk.0.attn_gate.weight", 6144, 32),
         ("blk.0.ssm_conv1d.weight", 10240, 1), ("blk.0.ssm_out.weight", 6144, 32), ("blk.0.ssm_a", 48, 32),
         ("blk.0.ssm_dt.bias", 48, 32), ("blk.0.ssm_alpha.weight", 48, 32), ("blk.0.ssm_beta.weight", 48, 32),
         ("blk.3.attn_q.weight", 12288, 32), ("blk.3.attn_k.weight", 1024, 32), ("blk.3.attn_v.weight", 1024, 32),
         ("blk.3.attn_output.weight", 6144, 32), ("blk.0.ffn_up.weight", 17408, 32),
         ("blk.0.ffn_gate.weight", 17408, 32), ("blk.0.ffn_down.weight", 17408, 32), ("cache_k_l3", 1024, 32),
         ("cache_v_l3", 1024, 32), ("cache_conv_l0", 10240, 32), ("cache_gdn_l0", 48, 32)]


@pytest.mark.parametrize("n_dev", [2, 4, 8])
def test_split_state_conserves_every_element(n_dev):  # split.rs:441-490 (extended to 4 and 8)
    for name, e, blck in CASES:
        st = tp.split_state(name, HP, e, blck, n_dev)
        assert extent(st, n_dev) == e, name
        assert all(v >= 0 for v in st.ne[:st.n_segments * n_dev]), name


def test_split_state_respects_granularity_and_balance():  # split.rs:492-518
    q = tp.split_state("blk.3.attn_q.weight", HP, 12288, 32, 2)
    assert q.ne[:2] == [6144, 6144]
    k = tp.split_state("blk.3.attn_k.weight", HP, 1024, 32, 2)
    assert k.ne[0] + k.ne[1] == 1024 and k.ne[0] % 256 == 0
    qkv = tp.split_state("blk.0.attn_qkv.weight", HP, 10240, 32, 2)
    assert qkv.n_segments == 1 and qkv.nr[0] == 5
    assert qkv.ne[0] + qkv.ne[1] == 2048 and qkv.ne[0] % 128 == 0
    up = tp.split_state("blk.0.ffn_up.weight", HP, 17408, 32, 2)
    assert up.ne[0] % 128 == 0 and up.ne[0] + up.ne[1] == 17408
    assert tp.split_state("blk.0.attn_norm.weight", HP, 5120, 1, 2).axis == tp.MIRRORED


def test_rotation_alternates_within_layer_kind():  # split.rs:520-532
    # rotation shows up as which device receives the leftover of an uneven split
    def owner_of_larger(name, e):
        st = tp.split_state(name, HP, e, 32, 2)
        return 0 if st.ne[0] >= st.ne[1] else 1
    # GDN layers 0,1,2 are the 1st/2nd/3rd recurrent layers -> rotation 0,1,0; an
    # uneven ffn_down extent (137 x 128) shows where the leftover lands
    odd = 17408 + 128
    assert [owner_of_larger(f"blk.{i}.ffn_down.weight", odd) for i in (0, 1, 2)] == [1, 0, 1]
    # attention layers 3 and 7 are the 1st/2nd attention layers -> rotation 0, 1
    a = owner_of_larger("blk.3.attn_output.weight", 6144 + 1536)
    b = owner_of_larger("blk.7.attn_output.weight", 6144 + 1536)
    assert a != b
    assert owner_of_larger("cache_k_l7", 1024 + 256) == owner_of_larger("blk.7.attn_k.weight", 1024 + 256)


def test_bad_arguments_fall_back_to_mirrored():  # meta.rs:47-64: never fails, degrades to MIRRORED
    assert tp.split_state("blk.0.ffn_up.weight", HP, 17408, 32, 0).axis == tp.MIRRORED
    assert tp.split_state("blk.0.ffn_up.weight", HP, -5, 32, 2).axis == tp.MIRRORED
    assert tp.split_state("", HP, 17408, 32, 2).axis == tp.MIRRORED
    assert tp.split_state("blk.x.ffn_up.weight", HP, 17408, 32, 2).axis == tp.MIRRORED


@pytest.mark.parametrize("n_dev", [1, 2, 4, 8])
def test_bench_stack_shards_line_up(n_dev):
    hp = tp.HP_BENCH_27B
    for il in range(4):
        sh = tp.layer_shards(hp, il, n_dev)
        for key, total in (("q", 6144), ("k", 1024), ("v", 1024), ("o", 6144), ("gate", 17408), ("down", 17408)):
            r = getattr(sh, key)
            assert r[0][0] == 0 and r[-1][1] == total and all(a <= b for a, b in r)
            assert all((b - a) % 256 == 0 for a, b in r), (key, r)   # whole Q4_K blocks
        assert sh.q == sh.o and sh.gate == sh.down


def test_bench_stack_tp8_follows_reference_granularity():
    # GQA groups stay whole (granularity n_gqa*head_k = 1536): at 8 devices only
    # four hold attention in a given layer, alternating by layer rotation
    hp = tp.HP_BENCH_27B
    s0 = tp.layer_shards(hp, 0, 8)
    s1 = tp.layer_shards(hp, 1, 8)
    assert [b - a for a, b in s0.q] == [0, 1536] * 4
    assert [b - a for a, b in s1.q] == [1536, 0] * 4
    assert sorted(b - a for a, b in s0.gate) == [2048] * 4 + [2304] * 4
