from mint_b200.main import app

app()
