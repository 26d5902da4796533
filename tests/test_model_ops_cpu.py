"""The on-disk layer loader of alveare_b200.model_ops (the reference's
blk.{l}.{proj}.weight_packed.npy files, runtime/py/model.py:38-52)."""
import numpy as np

from alveare_b200.model_ops import load_layer_weights


def test_load_layer_weights_reads_reference_file_names(tmp_path):
    a = np.arange(40, dtype=np.uint8).reshape(2, 20)
    np.save(tmp_path / "blk.2.ffn_up.weight_packed.npy", a)
    np.save(tmp_path / "blk.2.attn_q.weight_packed.npy", a + 1)
    got = load_layer_weights(tmp_path, 2)
    assert sorted(got) == ["attn_q", "ffn_up"] and np.array_equal(got["ffn_up"], a)
    assert load_layer_weights(tmp_path, 3) == {}
