"""`python -m offload.mobile.main` -> appcorr_b200.mobile.main."""
from appcorr_b200.mobile.main import main, run_mobile  # noqa: F401

if __name__ == "__main__":
    main()
