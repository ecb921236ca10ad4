"""On-device Q8_0 / Q4_0 quantization (esm_quantize_device) and the loaders that use it
(esm_load_host_quantized, esm_load_file_quantized): the blocks must be byte-identical to the host
quantizers (themselves pinned to the reference's BlockQ8_0/BlockQ4_0::quantize by the CPU tests),
and a model quantized on the device must produce exactly the logits of the same model quantized
on the host (EsmWeights::quantize_q8 / quantize_q4 then load). For Q3_LUT (EsmWeights::quantize_q3)
the fc1 / fc2 blocks come from the host quantizer and the attention matrices, which that model
keeps in Q4_0, from the device one."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def edge_blocks(rng):
    blocks = [
        np.zeros(32),                                  # d = 0: Q8 all zero, Q4 all 0x88
        np.full(32, -2.0),                             # constant negative block
    ]
    b = rng.standard_normal(32)
    b[5], b[17] = 3.0, -3.0                            # equal magnitudes: the first one sets the Q4 sign
    blocks.append(b)
    b = rng.standard_normal(32)
    b[9] = -7.5                                        # negative extreme
    blocks.append(b)
    # x / d lands exactly halfway between integers (round half away from zero).
    blocks.append(np.array([127.0] + [k + 0.5 for k in range(-16, 15)], dtype=np.float64))
    blocks.append(np.array([-8.0] + [k + 0.5 for k in range(-8, 7)] * 2 + [0.5], dtype=np.float64))
    blocks.append(np.full(32, 1e-41) * np.linspace(-1, 1, 32))   # subnormal: 1/d overflows for Q4
    blocks.append(rng.standard_normal(32) * 1e30)
    b = rng.standard_normal(32)
    b[3] = np.nan
    blocks.append(b)
    b = rng.standard_normal(32)
    b[11] = np.inf
    blocks.append(b)
    return np.concatenate(blocks).astype(np.float32)


@pytest.mark.parametrize("dtype_name", ["DTYPE_Q8_0", "DTYPE_Q4_0"])
def test_device_quantizer_matches_host(esm, dtype_name):
    import torch

    dtype = getattr(esm, dtype_name)
    rng = np.random.default_rng(7)
    x = np.concatenate([
        edge_blocks(rng),
        (rng.standard_normal(1 << 20) * 0.02).astype(np.float32),
        (rng.standard_normal(1 << 16) * rng.choice([1e-3, 1.0, 50.0], 1 << 16)).astype(np.float32),
    ])
    host = esm.quantize_q8(x) if dtype == esm.DTYPE_Q8_0 else esm.quantize_q4(x)
    src = torch.from_numpy(x).cuda()
    dst = torch.full((host.size,), 0xAB, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()
    esm.quantize_device(dtype, src.data_ptr(), x.size, dst.data_ptr(), stream.cuda_stream)
    torch.cuda.synchronize()
    dev = dst.cpu().numpy()
    bad = np.flatnonzero(dev != host)
    assert bad.size == 0, f"{bad.size} bytes differ, first at byte {bad[:4]}"


def test_device_quantizer_rejects_bad_arguments(esm):
    import torch

    src = torch.zeros(64, dtype=torch.float32, device="cuda")
    dst = torch.zeros(72, dtype=torch.uint8, device="cuda")
    with pytest.raises(esm.EsmError):
        esm.quantize_device(esm.DTYPE_Q8_0, src.data_ptr(), 63, dst.data_ptr())  # not a multiple of 32
    with pytest.raises(esm.EsmError):
        esm.quantize_device(esm.DTYPE_FP32, src.data_ptr(), 64, dst.data_ptr())  # not a block type
    with pytest.raises(esm.EsmError):
        esm.quantize_device(esm.DTYPE_Q8_0, src.data_ptr() + 4, 32, dst.data_ptr())  # src not 16-byte aligned


@pytest.mark.parametrize("dtype_name,shape", [("DTYPE_Q8_0", "esm2_35m"), ("DTYPE_Q4_0", "esm2_650m"),
                                              ("DTYPE_Q3_LUT", "esm2_150m")])
def test_device_quantized_model_matches_host_quantized(esm, tmp_path, dtype_name, shape):
    dtype = getattr(esm, dtype_name)
    base = getattr(esm, shape)()
    cfg = esm.EsmConfig(base.dim, base.hidden_dim, 2, base.n_heads, arch=base.arch)
    t32 = esm.synth_fp32_tensors(cfg, seed=5, bias_std=0.02, ln_jitter=0.1)
    lens = [9, 70, 131]
    seqs = esm.random_sequences(len(lens), lens, seed=6)

    def run(load):
        m = esm.Model(0)
        load(m)
        m.reserve(sum(lens), len(lens), max(lens))
        out = m.forward(seqs, want_hidden=True)
        m.close()
        return out

    ref = run(lambda m: m.load_tensors(cfg, dtype, esm.quantize_tensors(t32, dtype)))
    dev = run(lambda m: m.load_tensors_quantized(cfg, dtype, t32))
    np.testing.assert_array_equal(dev["logits"], ref["logits"])
    np.testing.assert_array_equal(dev["hidden"], ref["hidden"])

    # The same through an FP32 weights file (the reference's --q8 / --q4 load path); header-less
    # grouped_canonical_v1, since a CODQ header pins the preset layer count.
    path = tmp_path / "weights_fp32.bin"
    with open(path, "wb") as f:
        for n in esm.TENSOR_NAMES:
            f.write(np.ascontiguousarray(t32[n], dtype=np.float32).tobytes())
    viafile = run(lambda m: m.load_file_quantized(str(path), dtype, cfg))
    np.testing.assert_array_equal(viafile["logits"], ref["logits"])
