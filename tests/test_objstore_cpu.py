from marin_experiments_b200.utils.objstore import s3_spec, storage_options


def test_path_and_virtual_hosted():
    env = {"AWS_ENDPOINT_URL": "https://cwobject.com"}
    s = s3_spec("s3://bkt/a/b.bin", env)
    assert s["addressing"] == "path" and s["object_url"] == "https://cwobject.com/bkt/a/b.bin"
    env["LEVANTER_S3_VIRTUAL_HOSTED"] = "1"
    v = s3_spec("s3://bkt/a/b.bin", env)
    assert v["bucket"] == "" and v["endpoint"] == "https://bkt.cwobject.com" and v["key"] == "a/b.bin"
    assert storage_options("s3://bkt/x", env)["config_kwargs"]["s3"]["addressing_style"] == "virtual"
    assert s3_spec("s3://bkt/k", {})["object_url"] == "s3://bkt/k"
