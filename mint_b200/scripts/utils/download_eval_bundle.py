"""``mint download-eval``: fetch and unpack the CORE eval bundle into ``data/`` (scripts/utils/download_eval_bundle.py)."""

from __future__ import annotations

import shutil
import urllib.request
import zipfile
from pathlib import Path

URL = "https://karpathy-public.s3.us-west-2.amazonaws.com/eval_bundle.zip"


def main() -> None:
    Path("data").mkdir(exist_ok=True)
    Path("dump").mkdir(exist_ok=True)
    fname = "eval_bundle.zip"
    urllib.request.urlretrieve(URL, fname)  # noqa: S310
    with zipfile.ZipFile(fname) as zf:
        zf.extractall("data")
    shutil.move(fname, "dump/eval_bundle.zip")


if __name__ == "__main__":
    main()
