"""Generate the committed golden fixtures under tests/golden/.

Run in the build container, where the TabInfer checkout is mounted:

    python tests/golden/make_golden.py /path/to/TabInfer

What pins what:

* ternary_packs.npz -- codes/scales produced by the REFERENCE'S OWN numpy
  packer, native/tools/pack_bin.py:19-29 (pack_ternary), imported from the
  checkout and executed here, on
    - the tern.rs test fixtures (xorshift seeds 0x2026_0805+K and 0xC0FFEE+K,
      native/crates/n2-kernels/src/tern.rs:382-389, 405-435),
    - the n2 selftest fixtures (seed 0x9E3779B97F4A7C15, n2-cli main.rs:93-114),
    - config-1-style ternary weights (p=1/3 each code, f16-representable
      scales U(0.01,0.05)).
  The weights themselves are not stored: tests regenerate them from the seed,
  which also pins the xorshift generator.
* int4_js.npz -- int4 G=32 packs/scales from a second, independent numpy
  restatement of models/qwen3.js:3357-3426 (quantizeInt4Bf16 with the JS
  double / Float32Array / f32ToF16 round-half-up semantics).  No JavaScript
  runtime exists in this image, so the JS itself cannot be executed; this file
  cross-checks the C oracle against different code written from the same
  reference lines, on the self-test fixtures (qwen3.js:3077-3157) and edge
  cases (all-zero groups, scale underflow, negative zero, large values).
* tiny.cpu.bin + tiny_bin_weights.npz -- a `.cpu.bin` container written by the
  REFERENCE'S OWN writer, native/tools/pack_bin.py:31-75 (main), run on a
  synthetic two-shard safetensors checkpoint of Bonsai tensor names (f16
  embedding and norms, bf16 ternary projections and lm_head, seeded); the npz
  holds the checkpoint's raw 16-bit tensors.  It pins the device loader
  (tb_bin_open) against the format's own writer.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

import oracle  # noqa: E402  (fixture generators only: xorshift + ternaryish)


def js_f32_to_f16(f32):
    """Vectorised qwen3.js:3357-3374 over an f32 array."""
    x = np.ascontiguousarray(f32, np.float32).view(np.uint32).astype(np.int64)
    sign = (x >> 16) & 0x8000
    ex = (x >> 23) & 0xFF
    mant = x & 0x7FFFFF
    e = ex - 127 + 15
    out = np.zeros_like(x)
    # normal
    half = (e << 10) | (mant >> 13)
    half = half + ((mant >> 12) & 1)
    out = np.where((e > 0) & (e < 31), sign | half, out)
    # overflow
    out = np.where((e >= 31) & (ex != 0xFF), sign | 0x7C00, out)
    # inf / nan
    out = np.where(ex == 0xFF, sign | np.where(mant != 0, 0x7E00, 0x7C00), out)
    # subnormal / zero
    m = mant | 0x800000
    shift = np.clip(14 - e, 1, 62)
    sub = (m >> shift) + ((m >> (shift - 1)) & 1)
    out = np.where((e <= 0) & (e >= -10), sign | sub, out)
    out = np.where(e < -10, sign, out)
    return out.astype(np.uint16)


def js_quant_int4(u16, N, K):
    """Vectorised quantizeInt4Bf16, qwen3.js:3405-3426."""
    w = (u16.astype(np.uint32) << 16).view(np.float32).astype(np.float64).reshape(N, K // 32, 32)
    a = np.abs(w)
    a = np.where(np.isnan(a), 0.0, a)                       # NaN never wins `v > maxabs`
    maxabs = a.max(axis=2)
    scale = np.where(maxabs > 0, maxabs / 7.0, 1e-8)
    sbits = js_f32_to_f16(scale.astype(np.float32))
    sval = sbits.view(np.float16).astype(np.float64)
    with np.errstate(divide="ignore", invalid="ignore"):
        inv = 1.0 / sval
        prod = w * inv[:, :, None]
    fl = np.floor(prod)
    with np.errstate(invalid="ignore"):
        q = np.where(prod - fl >= 0.5, fl + 1.0, fl)
    q = np.where(np.isinf(prod), prod, q)
    q = np.clip(q, -8, 7)
    nib = np.where(np.isnan(q), 0, q + 8).astype(np.uint32).reshape(N, K)
    pack = np.zeros((N, K // 8), np.uint32)
    for i in range(8):
        pack |= nib[:, i::8] << np.uint32(4 * i)
    return pack, sbits.reshape(N, K // 32)


def int4_cases():
    cases = {}
    # qwen3.js:3077-3091 gemvQ fixture: W = cos(0.013 i), N=130, K=256
    i = np.arange(130 * 256, dtype=np.float64)
    cases["selftest_gemvQ"] = oracle.f32_to_bf16_trunc(np.cos(i * 0.013).astype(np.float32)).reshape(130, 256)
    # qwen3.js:3093-3106 gemvDP4A fixture: N=200, K=320
    i = np.arange(200 * 320, dtype=np.float64)
    cases["selftest_gemvDP4A"] = oracle.f32_to_bf16_trunc(np.cos(i * 0.013).astype(np.float32)).reshape(200, 320)
    # qwen3.js:3143-3157 gateUpSiluQ fixture up matrix: sin(0.009 i), I=130, H=256
    i = np.arange(130 * 256, dtype=np.float64)
    cases["selftest_up"] = oracle.f32_to_bf16_trunc(np.sin(i * 0.009).astype(np.float32)).reshape(130, 256)
    # config 2/3 distribution: N(0, 0.02) truncated to bf16
    rng = np.random.default_rng(20261201)
    cases["normal_002"] = oracle.f32_to_bf16_trunc(rng.normal(0, 0.02, (64, 1024)).astype(np.float32))
    # edge cases, one group per row of 32
    e = np.zeros((8, 64), np.float32)
    e[1, :32] = 1e-30                                     # scale underflows f16 -> q from +-Inf
    e[1, 32:] = -1e-30
    e[2, :] = -0.0                                        # negative zeros
    e[3, :] = np.linspace(-70000, 70000, 64)              # scale overflows? maxabs/7 = 10000 (fits)
    e[4, :] = np.linspace(-1, 1, 64) * 7.0                # exact halves at the quantization grid
    e[5, ::2] = 3.5
    e[5, 1::2] = -3.5
    e[6, :] = 2.0 ** -20 * np.arange(64)                  # subnormal f16 scales
    e[7, :] = np.float32(1e-7) * (np.arange(64) - 31.5)
    cases["edges"] = oracle.f32_to_bf16_trunc(e)
    return cases


def ternary_cases(pack_ternary_ref):
    out = {}
    shapes = [("tern_rs_oracle", 0x2026_0805, [(1, 64), (3, 128), (17, 256), (8, 1024)]),
              ("tern_rs_avx2", 0xC0FFEE, [(1, 64), (1, 192), (5, 192), (17, 256), (64, 2048)])]
    for tag, base, dims in shapes:
        for n, k in dims:
            _, _, _, _, w, _ = oracle.tern_fixture(n, k, base + k)
            codes, scales = pack_ternary_ref(w)
            out[f"{tag}_{n}x{k}_codes"] = codes
            out[f"{tag}_{n}x{k}_scales"] = scales
    for n, k in [(1, 64), (3, 192), (17, 256), (64, 2048)]:
        _, _, _, _, w, _ = oracle.tern_fixture(n, k, 0x9E3779B97F4A7C15)
        codes, scales = pack_ternary_ref(w)
        out[f"selftest_{n}x{k}_codes"] = codes
        out[f"selftest_{n}x{k}_scales"] = scales
    # config-1 style: codes uniform over {-1,0,+1}, f16-representable scales
    rng = np.random.default_rng(0x2026_1201)
    n, k = 96, 2048
    c = rng.integers(0, 3, (n, k)).astype(np.float32) - 1.0
    s = rng.uniform(0.01, 0.05, (n, k // 64)).astype(np.float16).astype(np.float32)
    w = c * np.repeat(s, 64, axis=1)
    # a group whose codes are all zero has max|w| = 0: keep one so the edge is pinned
    w[0, :64] = 0.0
    out["config1_w"] = w.astype(np.float32)
    codes, scales = pack_ternary_ref(w)
    out["config1_codes"] = codes
    out["config1_scales"] = scales
    return out


def _write_safetensors(path, tensors):
    """tensors: name -> (dtype str, shape, uint16 array)"""
    import json
    import struct
    hdr, off, blobs = {}, 0, []
    for name, (dt, shape, u16) in tensors.items():
        b = np.ascontiguousarray(u16, np.uint16).tobytes()
        hdr[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [off, off + len(b)]}
        off += len(b)
        blobs.append(b)
    h = json.dumps(hdr).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def tiny_checkpoint(seed=0xB1F):
    """Bonsai-named tensors: ternary bf16 projections (per-64 bf16 scales),
    f16 embedding and norms."""
    rng = np.random.default_rng(seed)
    H, V, I = 128, 96, 192

    def tern_bf16(N, K):
        s = (rng.uniform(0.01, 0.05, (N, K // 64)).astype(np.float32).view(np.uint32) & 0xFFFF0000).view(np.float32)
        w = rng.integers(-1, 2, (N, K)).astype(np.float32) * np.repeat(s, 64, axis=1)
        return (w.view(np.uint32) >> 16).astype(np.uint16)

    def f16(shape, lo, hi):
        return rng.uniform(lo, hi, shape).astype(np.float16).view(np.uint16)

    shard1 = {"model.embed_tokens.weight": ("F16", (V, H), f16((V, H), -1, 1)),
              "model.norm.weight": ("F16", (H,), f16((H,), 0.5, 1.5)),
              "model.layers.0.input_layernorm.weight": ("F16", (H,), f16((H,), 0.5, 1.5)),
              "model.layers.0.self_attn.q_proj.weight": ("BF16", (H, H), tern_bf16(H, H))}
    shard2 = {"model.layers.0.mlp.down_proj.weight": ("BF16", (H, I), tern_bf16(H, I)),
              "lm_head.weight": ("BF16", (V, H), tern_bf16(V, H))}
    return shard1, shard2


def bin_container(pack_bin):
    import json
    import tempfile
    shard1, shard2 = tiny_checkpoint()
    with tempfile.TemporaryDirectory() as d:
        _write_safetensors(os.path.join(d, "model-00001-of-00002.safetensors"), shard1)
        _write_safetensors(os.path.join(d, "model-00002-of-00002.safetensors"), shard2)
        wm = {n: "model-00001-of-00002.safetensors" for n in shard1}
        wm.update({n: "model-00002-of-00002.safetensors" for n in shard2})
        json.dump({"weight_map": wm}, open(os.path.join(d, "model.safetensors.index.json"), "w"))
        pack_bin.ROOT = d
        pack_bin.OUT = os.path.join(HERE, "tiny.cpu.bin")
        pack_bin.main()
    np.savez_compressed(os.path.join(HERE, "tiny_bin_weights.npz"),
                        **{n.replace(".", "__"): u16 for n, (_, _, u16) in {**shard1, **shard2}.items()})


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("TABINFER_REF", "")
    tools = os.path.join(ref, "native", "tools")
    if not os.path.exists(os.path.join(tools, "pack_bin.py")):
        sys.exit("usage: make_golden.py <TabInfer checkout>  (native/tools/pack_bin.py not found)")
    sys.path.insert(0, tools)
    import pack_bin  # the reference's own packer (module import only sets path constants)

    bin_container(pack_bin)

    tern = ternary_cases(pack_bin.pack_ternary)
    np.savez_compressed(os.path.join(HERE, "ternary_packs.npz"), **tern)

    int4 = {}
    for name, u16 in int4_cases().items():
        N, K = u16.shape
        pack, sc = js_quant_int4(u16, N, K)
        int4[name + "_w"] = u16
        int4[name + "_pack"] = pack
        int4[name + "_scales"] = sc
    np.savez_compressed(os.path.join(HERE, "int4_js.npz"), **int4)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
