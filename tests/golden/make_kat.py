"""Extract the reference crate's own known-answer tests into tests/golden/kat.json.

The reference (eclipse005/qwen3-aligner-wgpu) is Rust and cannot be built
here, so its unit-test tables are read as text from its test modules:

  src/align_input.rs:269-324   conv3_length / audio_token_count / padded_mel_frames
  src/postprocess.rs:155-241   fix_timestamps and pairing
  src/mel.rs:249-267           Hann window, reflection padding
  src/words.rs:235-...         split_words (Japanese cases skipped: nagisa)
  src/half16.rs:114-125        bf16 rounding of 0.1
  src/mrope.rs:95-117          dim-map layouts
  src/local_head.rs:1136-1207  Local Head primitives (Hann, mel bank, bands,
                               duration mask, overlap and duration repair)

Usage: python tests/golden/make_kat.py [REFERENCE_ROOT]
(REFERENCE_ROOT defaults to the path in $QA_REFERENCE_ROOT.)  The output is
committed; tests read only kat.json and never the reference tree.
"""
import json
import os
import re
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def _nums(s):
    return [int(x.replace("_", "")) for x in re.findall(r"-?[\d_]+", s)]


def main(root):
    src = lambda f: open(os.path.join(root, "src", f), encoding="utf-8").read()
    kat = {"source": "eclipse005/qwen3-aligner-wgpu unit tests (read as text)"}

    ai = src("align_input.rs")
    tests = ai[ai.index("#[cfg(test)]"):]
    kat["conv3_length"] = [[int(a), int(b)] for a, b in
                           re.findall(r"assert_eq!\(conv3_length\((\d+)\),\s*(\d+)\)", tests)]
    block = tests[tests.index("fn audio_token_count_over_sample_counts"):]
    block = block[block.index("let cases = ["):block.index("];")]
    pairs = re.findall(r"\(([\d_]+)(?:usize)?,\s*([\d_]+)(?:usize)?\)", block)
    kat["audio_token_count_samples"] = [[int(a.replace("_", "")), int(b.replace("_", ""))]
                                        for a, b in pairs]
    kat["padded_mel_frames"] = [[int(a), int(b), int(c)] for a, b, c in re.findall(
        r"assert_eq!\(padded_mel_frames\((\d+),\s*(\d+)\),\s*(\d+)\)", tests)]

    pp = src("postprocess.rs")
    tests = pp[pp.index("#[cfg(test)]"):]
    fx = []
    for m in re.finditer(r"let data = \[([^\]]*)\];(.*?)(?=\n    #\[test\]|\Z)", tests, re.S):
        data = _nums(m.group(1).replace("i64", ""))
        body = m.group(2)
        e = re.search(r"assert_eq!\(fix_timestamps\(&data\),\s*vec!\[([^\]]*)\]\)", body)
        if e:
            fx.append({"data": data, "want": _nums(e.group(1))})
        elif "fix_timestamps(&data), data.to_vec()" in body:
            fx.append({"data": data, "want": data})
        elif "windows(2).all" in body:
            fx.append({"data": data, "monotonic": True})
    kat["fix_timestamps"] = fx
    kat["pair_words"] = {"words": ["a", "b"], "raw": [2000, 2080, 2080, 2240],
                         "want": [["a", 2.0, 2.08], ["b", 2.08, 2.24]]}
    assert "decode_timestamps(&words, &[2000, 2080, 2080, 2240])" in tests

    mel = src("mel.rs")
    tests = mel[mel.index("#[cfg(test)]"):]
    rp = []
    for m in re.finditer(r"reflection_pad\(&signal, (\d+)\)(?:;\s*assert_eq!\(padded,\s*vec!\[|,\s*vec!\[)"
                         r"([^\]]*)\]", tests):
        rp.append({"signal": [1.0, 2.0, 3.0], "pad": int(m.group(1)),
                   "want": [float(x) for x in
                            re.findall(r"[\d.]+", m.group(2).replace("f32", ""))]})
    kat["reflection_pad"] = rp
    kat["hann4"] = {"n": 4, "w0": 0.0, "w2": 1.0, "tol": 1e-6}

    words = src("words.rs")
    tests = words[words.index("#[cfg(test)]"):]
    sp = []
    for m in re.finditer(r'split_words\(\s*"((?:[^"\\]|\\.)*)",\s*(Some\("(\w+)"\)|None)\s*\)\s*'
                         r'\.unwrap\(\),\s*vec!\[([^\]]*)\]', tests):
        lang = m.group(3)
        if lang in ("Japanese", "ja"):
            continue
        text = re.sub(r"\\u\{([0-9a-fA-F]+)\}", lambda k: chr(int(k.group(1), 16)), m.group(1))
        want = re.findall(r'"((?:[^"\\]|\\.)*)"', m.group(4))
        sp.append({"text": text, "language": lang, "want": want})
    kat["split_words"] = sp

    h16 = src("half16.rs")
    assert "assert_eq!(bf.to_bits(), 0x3DCD);" in h16
    kat["bf16_bits"] = [[0.1, 0x3DCD]]

    mr = src("mrope.rs")
    assert "build_dim_map(&[2, 1], 4, false)" in mr and "vec![0, 0, 1, 1]" in mr
    kat["dim_map"] = [{"section": [2, 1], "half": 4, "interleaved": False, "want": [0, 0, 1, 1]},
                      {"section": [24, 20, 20], "half": 64, "interleaved": True,
                       "prefix": [0, 1, 2, 0, 1, 2], "counts": [24, 20, 20]}]
    lh = src("local_head.rs")
    tests = lh[lh.index("#[cfg(test)]"):]
    m = re.search(r"np\.hanning\((\d+)\)\.astype\(np\.float32\)\[([\d, ]+)\]\s*\n\s*//\s*->\s*([\d., ]+)",
                  tests)
    idx = [int(x) for x in m.group(2).split(",")]
    vals = [float(x) for x in m.group(3).split(",")]
    assert "(w[10] - w[389]).abs() < 1e-6" in tests
    kat["lh_hann"] = {"n": int(m.group(1)), "index": idx, "want": vals, "tol": 1e-6,
                      "symmetric": [10, 389]}
    assert "(total - 1.0).abs() < 1e-5" in tests
    kat["lh_mel_bank"] = {"rows": 80, "bins": 257, "row_sum_tol": 1e-5}
    m = re.search(r"assert_eq!\(band_edges\((\d+)\),\s*\[([\d, ]+)\]\)", tests)
    kat["lh_band_edges"] = {"bins": int(m.group(1)), "want": _nums(m.group(2))}
    kat["lh_valid_class_count"] = [
        [float(a), int(b), int(c)] for a, b, c in re.findall(
            r"assert_eq!\(valid_class_count\(([\d.e]+),\s*(\d+)\),\s*(\d+)\)", tests)]
    pair = r"vec!\[\[([\d.]+), ([\d.]+)\], \[([\d.]+), ([\d.]+)\]\]"
    kat["lh_remove_overlaps"] = [
        {"intervals": [[float(g[0]), float(g[1])], [float(g[2]), float(g[3])]],
         "want": [[float(g[4]), float(g[5])], [float(g[6]), float(g[7])]]}
        for g in re.findall(r"let mut v = " + pair + r";\s*remove_neighbor_overlaps\(&mut v\);"
                            r"\s*assert_eq!\(v, " + pair + r"\)", tests)]
    bd = re.findall(r"let mut v = " + pair + r";\s*bound_to_duration\(&mut v, ([\d.]+)\);", tests)
    assert len(bd) == 2 and "assert!((v[1][1] - 10.0).abs() < 1e-9" in tests
    kat["lh_bound_to_duration"] = [
        {"intervals": [[float(g[0]), float(g[1])], [float(g[2]), float(g[3])]],
         "duration_ms": float(g[4]), "want": [[float(g[0]), float(g[1])], [float(g[2]), float(g[3])]]}
        for g in bd[:1]] + [
        {"intervals": [[float(g[0]), float(g[1])], [float(g[2]), float(g[3])]],
         "duration_ms": float(g[4]), "last_end": 10.0, "min_len": 5.0, "tol": 1e-9}
        for g in bd[1:]]
    with open(os.path.join(HERE, "kat.json"), "w", encoding="utf-8") as f:
        json.dump(kat, f, indent=1, ensure_ascii=False)
    print({k: len(v) if isinstance(v, list) else 1 for k, v in kat.items()})


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("QA_REFERENCE_ROOT", ""))
