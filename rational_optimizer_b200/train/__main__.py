"""``python -m rational_optimizer_b200.train``: the language-model trainer."""
import sys

from .trainer import main

sys.exit(main())
