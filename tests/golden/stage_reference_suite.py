"""Stage the reference's own test files for an unmodified run against
thork_b200 (``tests/test_gpu_reference_suite.py``).

    python tests/golden/stage_reference_suite.py [/path/to/reference]

Copies ``tests/test_thork.py`` and ``tests/test_kittens.py`` of the
reference checkout, byte for byte, into ``tests/_reference_suite/``.  That
folder is git-ignored: the files are never committed to this repository,
they only travel with the working tree to the GPU machine, where the
reference checkout is absent.  ``__graft_entry__.build()`` calls this when
the reference checkout is present.  A SHA-256 of each staged file is written
beside it so the GPU test can show it ran the files unmodified.
"""

import hashlib
import json
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
TESTS = os.path.dirname(HERE)
STAGE = os.path.join(TESTS, "_reference_suite")
FILES = ("test_thork.py", "test_kittens.py")
DEFAULT_REF = "/root/reference"


def stage(ref_root: str = DEFAULT_REF) -> bool:
    """Copy the files; False (and nothing written) when the checkout is absent."""
    src_dir = os.path.join(ref_root, "tests")
    if not all(os.path.isfile(os.path.join(src_dir, f)) for f in FILES):
        return False
    os.makedirs(STAGE, exist_ok=True)
    digests = {}
    for f in FILES:
        dst = os.path.join(STAGE, f)
        shutil.copyfile(os.path.join(src_dir, f), dst)
        with open(dst, "rb") as fh:
            digests[f] = hashlib.sha256(fh.read()).hexdigest()
    with open(os.path.join(STAGE, "SHA256.json"), "w") as fh:
        json.dump({"source": os.path.abspath(src_dir), "sha256": digests}, fh, indent=1)
    return True


if __name__ == "__main__":
    ok = stage(sys.argv[1] if len(sys.argv) > 1 else DEFAULT_REF)
    print("staged" if ok else "reference checkout not found; nothing staged")
