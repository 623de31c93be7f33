import os

import numpy as np

from b200infer import gguf as G


def test_round_trip(tmp_path):
    cfg = G.Qwen3Config(n_vocab=64, n_embd=32, n_layer=2, n_head=2, n_head_kv=1, head_dim=16, n_ff=48,
                        n_ctx_train=128, tied=False)
    path = os.path.join(tmp_path, "m.gguf")
    over = {"blk.1.ffn_up.weight": np.arange(48 * 32, dtype=np.float32).reshape(48, 32)}
    G.write_gguf(path, cfg, seed=3, tensors=over)
    rd = G.GGUFReader(path)
    assert rd.config() == G.Qwen3Config(**{**cfg.as_dict(), "rms_eps": rd.config().rms_eps})
    assert abs(rd.config().rms_eps - 1e-6) < 1e-12
    names = [n for n, _, _ in G.tensor_specs(cfg)]
    assert rd.names() == names and "output.weight" in names
    assert np.array_equal(rd.tensor("blk.1.ffn_up.weight"), over["blk.1.ffn_up.weight"])
    assert np.all(rd.tensor("blk.0.attn_norm.weight") == 1.0)
    w = rd.tensor("blk.0.attn_q.weight")
    assert w.shape == (32, 32) and abs(float(w.std()) - 0.02) < 0.005
    assert np.array_equal(w, G.seeded_tensor("blk.0.attn_q.weight", (32, 32), "mat", 3))
    for n in names:
        off = rd.infos[n][2]
        assert (rd.data_offset + off) % 64 == 0


def test_weight_bytes_per_token_matches_survey():
    # 28 layers x 62,914,560 + 28 x 9,216 (norms) + 622,329,856 (tied LM head) + 4,096
    assert G.QWEN3_0_6B.weight_bytes_per_token == 2_384_199_680
