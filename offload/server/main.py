"""`python -m offload.server.main` -> appcorr_b200.server.main."""
from appcorr_b200.server.main import main, run_server  # noqa: F401

if __name__ == "__main__":
    main()
