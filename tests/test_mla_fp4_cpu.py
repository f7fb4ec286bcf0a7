"""The NVFP4 latent cache row (vLLM's nvfp4_ds_mla layout) as the CPU statement writes and reads it.

Row of kv_lora Cl latent + R rope values: [0, Cl/2) e2m1 pairs (low nibble = even dim), [Cl/2, Cl/2 + R) the
rope in unscaled e4m3, then the Cl/16 e4m3 block scales with scale s at byte (Cl/64) * (s % 4) + s // 4 of
their region; 352 bytes at Cl 512, R 64 (reference: kernels-oxide/nvfp4_ds_mla/src/main.rs:11-20).  The GPU
writer is checked byte for byte against `mla_fp4_pack` in test_mla_gpu.py.
"""
import torch

from vllm_suffix_hybrid_b200 import ops
from vllm_suffix_hybrid_b200.ops import reference as ref


def test_row_sizes_and_scale_permutation():
    assert ops.mla_fp4_row_bytes(512, 64) == 352
    assert ops.mla_fp4_row_bytes(64, 64) == 112  # 100 bytes padded to 16
    pos = ref.mla_fp4_scale_pos(512)
    assert pos.tolist() == [8 * (s % 4) + s // 4 for s in range(32)]
    assert sorted(pos.tolist()) == list(range(32))
    assert ref.mla_fp4_scale_pos(64).tolist() == [0, 1, 2, 3]


def test_pack_places_codes_rope_and_scales():
    c = torch.zeros(1, 512)
    c[0, 80] = 2.0   # block 5: amax 12 / 6 -> scale 2 (e4m3 0x40); 2 / 2 = 1.0 -> code 2, even dim: low nibble
    c[0, 81] = -12.0  # -6.0 -> code 0xF, odd dim: high nibble
    c[0, 82] = 1.0    # 0.5 -> code 1
    kpe = torch.zeros(1, 64)
    kpe[0, 0] = 1000.0  # saturates at 448 (0x7E)
    kpe[0, 3] = -0.5    # 0xB0
    rows = ref.mla_fp4_pack(c, kpe)
    assert rows.shape == (1, 352) and rows.dtype == torch.uint8
    assert int(rows[0, 40]) == 0xF2 and int(rows[0, 41]) == 0x01
    assert int(rows[0, 256]) == 0x7E and int(rows[0, 259]) == 0xB0
    assert int(rows[0, 320 + 8 * 1 + 1]) == 0x40  # block 5 -> byte 8 (5 % 4) + 5 // 4 = 9
    assert int(rows[0, 320]) == 0x01  # an all-zero block keeps the 2^-9 floor scale (e4m3 0x01)
    vals = ref.mla_fp4_unpack(rows, 512, 64)
    assert vals[0, 80].item() == 2.0 and vals[0, 81].item() == -12.0 and vals[0, 82].item() == 1.0
    assert vals[0, 512].item() == 448.0 and vals[0, 515].item() == -0.5


def test_unpack_matches_quantise_dequantise():
    g = torch.Generator().manual_seed(3)
    for Cl, R in ((512, 64), (64, 64)):
        c = (torch.randn(40, Cl, generator=g) * torch.rand(40, 1, generator=g) * 3).to(torch.bfloat16)
        c[0, :16] = 0
        c[1, 16:32] = 1e-6  # below the floor scale's reach
        kpe = (torch.randn(40, R, generator=g) * 20).to(torch.bfloat16)
        rows = ref.mla_fp4_pack(c, kpe)
        want = torch.cat([ref.mla_fp4_qdq(c), ref.e4m3_qdq(kpe)], -1)
        assert torch.equal(ref.mla_fp4_unpack(rows, Cl, R), want)
        # half the widest e2m1 gap (4 -> 6) is one scale step; the e4m3 scale is within 1/16 of amax / 6
        amax = c.float().view(40, -1, 16).abs().amax(-1).repeat_interleave(16, 1)
        assert bool(((want[:, :Cl] - c.float()).abs() <= amax / 6 * (1 + 2 ** -4) + 2 ** -9).all())


def test_cpu_cache_write_stores_the_row_values():
    g = torch.Generator().manual_seed(5)
    c = torch.randn(6, 512, generator=g).to(torch.bfloat16)
    kpe = (torch.randn(6, 64, generator=g) * 4).to(torch.bfloat16)
    lat = torch.zeros(2, 64, 576)
    slots = torch.tensor([0, 5, 64, -1, 70, 127])
    ops.mla_cache_write(lat, c.float(), kpe.float(), slots, fp4=True)
    vals = ref.mla_fp4_unpack(ref.mla_fp4_pack(c, kpe), 512, 64)
    for i, s in enumerate(slots.tolist()):
        if s >= 0:
            assert torch.equal(lat[s // 64, s % 64], vals[i])


def test_deepseek_block_bytes_and_one_layer_mtp_cache():
    """The engine sizes a DeepSeek KV block from the model's own rows (latent + indexer page per layer), and
    the MTP draft allocates one layer of cache, not the target's whole stack."""
    from vllm_suffix_hybrid_b200.engine.config import deepseek_v32_config, shrink
    from vllm_suffix_hybrid_b200.models import deepseek

    cfg = shrink(deepseek_v32_config(), layers=3, hidden=128, vocab=512)
    cfg.kv_format = "nvfp4"  # on CPU the cache keeps the model dtype (it stores the values NVFP4 rows return)
    m, mtp = deepseek.build(cfg, "cpu", 0, True)
    per = m.kv_block_bytes(64)
    assert per == 64 * (cfg.kv_lora + cfg.qk_rope) * m.embed.element_size() + (
        ops.DSA_PAGE_BYTES if cfg.dsa_topk else 0)
    assert mtp.kv_block_bytes(64) == per
    lat, idx = mtp.allocate_caches(4, 64)
    assert lat.shape == (4, 64, cfg.kv_lora + cfg.qk_rope)
    assert len(m.allocate_caches(4, 64, 0, 0)) == 3
