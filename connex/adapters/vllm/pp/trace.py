"""``CONNEX_PP_TRACE`` step stamps under the reference's module path; the
implementation is :mod:`connex.pp.steptrace`."""
import sys

from connex.pp.steptrace import ON, flush, load, main, timeline, tr  # noqa: F401

if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
