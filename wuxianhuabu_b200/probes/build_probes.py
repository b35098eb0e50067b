"""Build the hardware probes (standalone CUDA programs) into wuxianhuabu_b200/probes/_build/.

Run on a B200: ``python -m wuxianhuabu_b200.probes.build_probes`` then e.g.
``wuxianhuabu_b200/probes/_build/mb_attn``. Each probe prints one line per case."""
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
PROBES = ["mb_attn", "mb_tma", "mb_smem", "mb_mufu"]


def main() -> None:
    out = HERE / "_build"
    out.mkdir(exist_ok=True)
    for name in PROBES:
        cmd = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-o", str(out / name),
               str(HERE / f"{name}.cu")]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.exit(f"{' '.join(cmd)}\n{r.stdout}{r.stderr}")
        print(out / name)


if __name__ == "__main__":
    main()
