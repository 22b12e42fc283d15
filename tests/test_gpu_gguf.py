"""GPU: MoE expert packs uploaded from a GGUF file (qw6cu_gguf_upload_moe)
run the routed MoE layer like packs made from the same bytes in memory, and
match the oracle's composition of qw6_apply_layer_moe (qw6.c:2246-2264)."""
import numpy as np
import pytest

from qw6_b200 import lib as L
from qw6_b200 import synth as S
from tests.conftest import rel_err
from tests.gguf_util import write_gguf
from tests.gpu_util import dev, empty_f32, host, sync

pytestmark = pytest.mark.gpu


def test_moe_from_gguf_upload(tmp_path, cuda, oracle, rng):
    E, H, I, K, T, layers = 16, 2048, 512, 8, 3, 2
    mats = {}
    tensors = []
    for l in range(layers):
        g, u, d = S.moe_weights(rng, E, S.Q4_K, S.Q6_K, H, I)
        mats[l] = (g, u, d)
        tensors += [(f"blk.{l}.ffn_gate_exps.weight", "Q4_K", [H, I, E], g),
                    (f"blk.{l}.ffn_up_exps.weight", "Q4_K", [H, I, E], u),
                    (f"blk.{l}.ffn_down_exps.weight", "Q6_K", [I, H, E], d)]
    path = tmp_path / "moe.gguf"
    write_gguf(path, tensors, [], alignment=32)
    gg = L.Gguf(path)
    tab = gg.upload_moe(cuda, layers)
    try:
        assert tab.n_layers == layers
        for l in range(layers):
            gp, up, dp = gg.layer_packs(tab, l)
            assert (gp.quant, up.quant, dp.quant) == (S.Q4_K, S.Q4_K, S.Q6_K)
            logits = rng.standard_normal((T, E), dtype=np.float32)
            x = rng.standard_normal((T, H), dtype=np.float32)
            ld, xd = dev(logits), dev(x)
            out = empty_f32(T, H)
            sync(cuda)
            cuda.moe_decode(gp, up, dp, ld.data_ptr(), xd.data_ptr(), out.data_ptr(), T, H, I, E, K)
            cuda.synchronize()
            got = host(out)
            g, u, d = mats[l]
            ref, _, _ = oracle.moe_layer(S.Q4_K, g, u, S.Q6_K, d, logits, x, top_k=K)
            for t in range(T):
                assert rel_err(got[t], ref[t]) <= 1e-3, (l, t)
    finally:
        gg.free_table(tab)
        gg.close()
