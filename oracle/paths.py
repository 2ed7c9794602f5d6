"""Where the oracle's inputs live (test infrastructure only).

reference_dir(): the tinytrain reference sources. Taken from the
TT_REFERENCE environment variable, else from _ref/reference_dir.txt, which
`make -C oracle REF=<dir>` writes when it builds the oracle. None when
neither names a directory holding the sources (e.g. on a machine that only
received the prebuilt oracle).

nlohmann_dir(): an include directory holding nlohmann/json.hpp (3.11.3,
the version the reference pins), needed to compile the reference's
model.cpp. Taken from TT_NLOHMANN, else from the copy that the installed
cudnn frontend ships beside the Python cudnn package. None if absent.
"""
from __future__ import annotations

import os

_HERE = os.path.dirname(os.path.abspath(__file__))


def _has_sources(d):
    return bool(d) and os.path.isdir(os.path.join(d, "src")) and \
        os.path.isdir(os.path.join(d, "include", "tinytrain"))


def reference_dir():
    d = os.environ.get("TT_REFERENCE")
    if _has_sources(d):
        return d
    try:
        with open(os.path.join(_HERE, "_ref", "reference_dir.txt")) as f:
            d = f.read().strip()
    except OSError:
        return None
    return d if _has_sources(d) else None


def nlohmann_dir():
    d = os.environ.get("TT_NLOHMANN")
    if d and os.path.exists(os.path.join(d, "nlohmann", "json.hpp")):
        return d
    try:
        import cudnn  # noqa: F401  (only its install location is used)
    except Exception:
        return None
    d = os.path.join(os.path.dirname(os.path.dirname(cudnn.__file__)), "include",
                     "cudnn_frontend", "thirdparty")
    return d if os.path.exists(os.path.join(d, "nlohmann", "json.hpp")) else None


if __name__ == "__main__":
    print(nlohmann_dir() or "")
