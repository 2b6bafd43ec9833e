"""`python -m kernelverify_b200.roofline`: measure and print the ceilings."""

import sys

from kernelverify_b200.roofline import main

sys.exit(main())
