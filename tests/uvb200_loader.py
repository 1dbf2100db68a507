"""Test-side access to the product package (see ultravec_ann_b200_loader)."""
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
from ultravec_ann_b200_loader import load  # noqa: E402,F401
