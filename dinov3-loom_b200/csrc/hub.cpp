// hub.cpp - the pinned weights in the shared Hugging Face cache (src/hub.rs), offline only: the
// path of the cached file is resolved the way the reference's client resolves it, and a miss is
// reported with the reference's message. This library has no network client, so a miss is an
// error whether or not downloads are allowed.
#include <sys/stat.h>

#include <cstdlib>
#include <cstring>
#include <string>

#include "dinov3.h"

namespace dv3 {

// src/hub.rs:6-11
constexpr const char *kHubOrg = "facebook";
constexpr const char *kHubName = "dinov3-vits16plus-pretrain-lvd1689m";
constexpr const char *kHubRevision = "c93d816fc9e567563bc068f01475bec89cc634a6";
constexpr const char *kHubFile = "model.safetensors";

static std::string env(const char *name) {
  const char *v = std::getenv(name);
  return v ? std::string(v) : std::string();
}

// The cache directory: HF_HUB_CACHE, else HF_HOME/hub, else XDG_CACHE_HOME/huggingface/hub,
// else ~/.cache/huggingface/hub (the Hugging Face clients' order).
static std::string hub_cache_dir() {
  if (!env("HF_HUB_CACHE").empty()) return env("HF_HUB_CACHE");
  if (!env("HF_HOME").empty()) return env("HF_HOME") + "/hub";
  if (!env("XDG_CACHE_HOME").empty()) return env("XDG_CACHE_HOME") + "/huggingface/hub";
  return env("HOME") + "/.cache/huggingface/hub";
}

// src/hub.rs:17-54. Returns true and the path when the pinned file is cached; otherwise false and
// the message the reference gives (offline: HF_HUB_OFFLINE set to anything but "" or "0", or the
// caller's flag).
bool hub_weights(bool offline, std::string *path, std::string *err) {
  const std::string off = env("HF_HUB_OFFLINE");
  offline = offline || (!off.empty() && off != "0");
  const std::string p = hub_cache_dir() + "/models--" + kHubOrg + "--" + kHubName + "/snapshots/" +
                        kHubRevision + "/" + kHubFile;
  struct stat st {};
  if (::stat(p.c_str(), &st) == 0 && S_ISREG(st.st_mode)) {  // follows the snapshot symlink
    *path = p;
    return true;
  }
  const std::string what = std::string(kHubOrg) + "/" + kHubName + " at " + kHubRevision;
  if (offline)
    *err = what + ": " + kHubFile + " is not cached and model downloads are disabled";
  else
    *err = std::string("cannot download ") + what + ": " + kHubFile +
           " (this library reads the Hugging Face cache only and has no network client)";
  return false;
}

}  // namespace dv3
