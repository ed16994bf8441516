"""``python -m oxidizr_b200`` == the ``oxidizr`` command."""
import sys

from .cli import main

sys.exit(main())
